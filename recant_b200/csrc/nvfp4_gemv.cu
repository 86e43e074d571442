// NVFP4 GEMM for a few rows of A (M <= 4): out[m, n] = sum_k A[m, k] B[n, k] * gA * gB, the same
// product as rb2_nvfp4_gemm (recant/model/nvfp4.py:108-125) for the decode step, where A is one token
// per sequence and the 128-row tiles of the tensor-core kernel would be almost empty. The work is
// reading B once (K/2 code bytes + K/16 scale bytes per row), so it is shaped for HBM:
//   * every CTA dequantizes A (e2m1 x e4m3, exact in fp32) into shared memory, 4 floats of padding
//     per 32 so that the lanes' float4 reads of one k-chunk fall in different banks;
//   * one warp per row of B: each lane streams 16-byte chunks of codes (32 elements, two scale
//     blocks), sums a * e2m1(b) per 16-element block and multiplies by the block's scale;
//   * a warp reduction per output, times gA gB, written as fp32 or bf16.
// Scales here are the row-major [rows, K/16] e4m3 bytes (FP4Tensor.scales), not the blocked layout.
#include <cuda_fp8.h>

#include "common.cuh"

namespace rb2 {
namespace {

constexpr int kMaxM = 4;
constexpr int kThreads = 256;
constexpr int kBatch = 4;  // 16-byte code chunks each lane has in flight

__device__ __forceinline__ float e2m1_value(uint32_t c) {
  // magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6; bit 3 is the sign
  const uint32_t i = c & 7u;
  const float v = i < 4 ? 0.5f * float(i) : (i == 4 ? 2.f : (i == 5 ? 3.f : (i == 6 ? 4.f : 6.f)));
  return (c & 8u) ? -v : v;
}

__host__ __device__ __forceinline__ int padded(int k) { return k + (k >> 5) * 4; }  // 4 floats after every 32

__global__ void __launch_bounds__(kThreads) nvfp4_gemv_kernel(const uint8_t* __restrict__ a_codes,
                                                              const uint8_t* __restrict__ a_scales,
                                                              const float* __restrict__ ga,
                                                              const uint8_t* __restrict__ b_codes,
                                                              const uint8_t* __restrict__ b_scales,
                                                              const float* __restrict__ gb, int M, int N, int K,
                                                              void* __restrict__ out, int out_bf16) {
  extern __shared__ __align__(16) float gsm[];
  float* t8 = gsm;             // e4m3 byte -> float
  float* t2 = gsm + 256;       // e2m1 code -> float
  float* ad = gsm + 256 + 16;  // A dequantized, [M][padded(K)]
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int kp = padded(K);
  {
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(tid), __NV_E4M3);
    t8[tid] = __half2float(__half(hr));
    if (tid < 16) t2[tid] = e2m1_value(tid);
  }
  __syncthreads();
  for (int m = 0; m < M; ++m)
    for (int k = tid; k < K; k += kThreads) {
      const uint32_t c = (a_codes[size_t(m) * (K / 2) + k / 2] >> (4 * (k & 1))) & 0xFu;
      ad[m * kp + padded(k)] = t2[c] * t8[a_scales[size_t(m) * (K / 16) + k / 16]];
    }
  __syncthreads();
  const float g = ga[0] * gb[0];
  const int warps = gridDim.x * (kThreads / 32);
  for (int n = blockIdx.x * (kThreads / 32) + w; n < N; n += warps) {
    const uint4* wr = reinterpret_cast<const uint4*>(b_codes + size_t(n) * (K / 2));
    const uint8_t* sr = b_scales + size_t(n) * (K / 16);
    float acc[kMaxM] = {0.f, 0.f, 0.f, 0.f};
    // up to kBatch chunks per lane in flight: chunk c holds elements 32c .. 32c + 31
    for (int cb = l; cb < K / 32; cb += 32 * kBatch) {
      uint4 u[kBatch];
      uint8_t sb[kBatch][2];
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int c = cb + 32 * i;
        if (c < K / 32) {
          u[i] = __ldg(wr + c);
          sb[i][0] = __ldg(sr + 2 * c);
          sb[i][1] = __ldg(sr + 2 * c + 1);
        }
      }
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int c = cb + 32 * i;
        if (c >= K / 32) break;
        const uint32_t words[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {  // two 16-element scale blocks
          const float sc = t8[sb[i][hb]];
          float bv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) bv[j] = t2[(words[2 * hb + j / 8] >> (4 * (j & 7))) & 0xFu];
#pragma unroll
          for (int m = 0; m < kMaxM; ++m) {
            if (m >= M) break;
            const float4* ap = reinterpret_cast<const float4*>(ad + m * kp + padded(32 * c + 16 * hb));
            float part = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 a4 = ap[q];
              part = fmaf(a4.x, bv[4 * q], part);
              part = fmaf(a4.y, bv[4 * q + 1], part);
              part = fmaf(a4.z, bv[4 * q + 2], part);
              part = fmaf(a4.w, bv[4 * q + 3], part);
            }
            acc[m] = fmaf(part, sc, acc[m]);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < kMaxM; ++m) {
      if (m >= M) break;
      float v = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (l == 0) {
        if (out_bf16) static_cast<__nv_bfloat16*>(out)[size_t(m) * N + n] = __float2bfloat16_rn(v * g);
        else static_cast<float*>(out)[size_t(m) * N + n] = v * g;
      }
    }
  }
}

size_t gemv_smem(int M, int K) { return size_t(256 + 16 + M * padded(K)) * 4; }

}  // namespace
}  // namespace rb2

using namespace rb2;

extern "C" int rb2_nvfp4_gemv(const uint8_t* a_codes, const uint8_t* a_scales, const float* a_gscale,
                              const uint8_t* b_codes, const uint8_t* b_scales, const float* b_gscale, int64_t M,
                              int64_t N, int64_t K, void* out, int out_dtype, void* stream) {
  RB2_CHECK_ARG(M >= 1 && M <= kMaxM && N >= 1 && K >= 32 && K % 32 == 0 && N < (int64_t(1) << 31) &&
                    K < (int64_t(1) << 24),
                "nvfp4_gemv: need 1 <= M <= %d, N >= 1 and K %% 32 == 0 (M=%lld N=%lld K=%lld)", kMaxM, (long long)M,
                (long long)N, (long long)K);
  RB2_CHECK_ARG(a_codes && a_scales && a_gscale && b_codes && b_scales && b_gscale && out, "nvfp4_gemv: null pointer");
  RB2_CHECK_ARG((reinterpret_cast<uintptr_t>(b_codes) & 15) == 0, "nvfp4_gemv: B codes must be 16-byte aligned");
  RB2_CHECK_ARG(out_dtype == RB2_F32 || out_dtype == RB2_BF16, "nvfp4_gemv: out_dtype");
  const size_t smem = gemv_smem(int(M), int(K));
  RB2_CHECK_ARG(smem <= 200 * 1024, "nvfp4_gemv: M x K = %lld x %lld does not fit in shared memory", (long long)M,
                (long long)K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 148;
  RB2_CUDA(cudaGetDevice(&dev), "nvfp4_gemv: device");
  RB2_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "nvfp4_gemv: SM count");
  RB2_CUDA(cudaFuncSetAttribute(nvfp4_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
           "nvfp4_gemv: smem attribute");
  const int64_t want = (N + kThreads / 32 - 1) / (kThreads / 32);
  const unsigned grid = unsigned(want < int64_t(sms) * 2 ? want : int64_t(sms) * 2);
  ProfScope ps_("nvfp4_gemv", s);
  nvfp4_gemv_kernel<<<grid, kThreads, smem, s>>>(a_codes, a_scales, a_gscale, b_codes, b_scales, b_gscale, int(M),
                                                  int(N), int(K), out, out_dtype == RB2_BF16);
  RB2_CHECK_LAUNCH("nvfp4_gemv");
  return RB2_OK;
}
