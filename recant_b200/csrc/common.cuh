// Shared helpers for the recant_b200 CUDA library (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/recant_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "recant_b200 kernels target sm_100a (B200) only"
#endif

namespace rb2 {

// ----- host-side error reporting -------------------------------------------------------------
void set_error(const char* fmt, ...);

#define RB2_CHECK_ARG(cond, ...)                 \
  do {                                           \
    if (!(cond)) {                               \
      ::rb2::set_error(__VA_ARGS__);             \
      return RB2_EINVAL;                         \
    }                                            \
  } while (0)

#define RB2_CHECK_LAUNCH(what)                                                       \
  do {                                                                               \
    cudaError_t e_ = cudaGetLastError();                                             \
    if (e_ != cudaSuccess) {                                                         \
      ::rb2::set_error("%s: %s", what, cudaGetErrorString(e_));                      \
      return (e_ == cudaErrorMemoryAllocation) ? RB2_ENOMEM : RB2_ECUDA;             \
    }                                                                                \
  } while (0)

#define RB2_CUDA(call, what)                                                         \
  do {                                                                               \
    cudaError_t e_ = (call);                                                         \
    if (e_ != cudaSuccess) {                                                         \
      ::rb2::set_error("%s: %s", what, cudaGetErrorString(e_));                      \
      return (e_ == cudaErrorMemoryAllocation) ? RB2_ENOMEM : RB2_ECUDA;             \
    }                                                                                \
  } while (0)

// ----- launch profiler (prof.cu): brackets one kernel launch with events when enabled ---------
class ProfScope {
 public:
  ProfScope(const char* name, cudaStream_t s);
  ~ProfScope();
  ProfScope(const ProfScope&) = delete;
  ProfScope& operator=(const ProfScope&) = delete;

 private:
  int slot_;
  cudaStream_t s_;
};

// ----- workspace carving -----------------------------------------------------------------------
// A bump allocator over a caller-provided device buffer; every region is 256-byte aligned.
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
  size_t bytes() const { return (off + 255) & ~size_t(255); }
};

// ----- element loads ---------------------------------------------------------------------------
__device__ __forceinline__ float ldf(const float* p) { return *p; }
__device__ __forceinline__ float ldf(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void stf(float* p, float v) { *p = v; }
__device__ __forceinline__ void stf(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace rb2
