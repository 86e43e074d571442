// Device self-test of the tcgen05 operand layouts (tc.cuh): one CTA computes D = A . B^T for a
// single tile with A and B in either K-major or MN-major SW128 shared-memory layout, so a layout or
// descriptor mistake shows up as a wrong product rather than inside a large kernel.
#include "tc.cuh"

namespace rb2 {
namespace {

__global__ void __launch_bounds__(128) selftest_mma_kernel(const __nv_bfloat16* __restrict__ A,
                                                           const __nv_bfloat16* __restrict__ B,
                                                           float* __restrict__ D, int a_mn, int b_mn, int M,
                                                           int N, int K, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // SW128 atoms must start on a 1024-byte boundary of the shared address space
  unsigned char* smem = smem_raw + ((1024 - (tc::smem_u32(smem_raw) & 1023)) & 1023);
  unsigned char* sa = smem;                      // up to 128 x 128 bf16 = 32 KB
  unsigned char* sb = smem + 32768;              // up to 128 x 128 bf16 = 32 KB
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x;
  // A(m, k): K-major -> tile rows = M, "k" = K;  MN-major -> tile rows = K, "k" = M
  for (int idx = tid; idx < M * K; idx += 128) {
    const int m = idx / K, k = idx % K;
    const __nv_bfloat16 x = a_mn ? A[k * M + m] : A[m * K + k];
    const uint32_t off = a_mn ? tc::sw128_offset(k, m, K) : tc::sw128_offset(m, k, M);
    *reinterpret_cast<__nv_bfloat16*>(sa + off) = x;
  }
  for (int idx = tid; idx < N * K; idx += 128) {
    const int n = idx / K, k = idx % K;
    const __nv_bfloat16 x = b_mn ? B[k * N + n] : B[n * K + k];
    const uint32_t off = b_mn ? tc::sw128_offset(k, n, K) : tc::sw128_offset(n, k, N);
    *reinterpret_cast<__nv_bfloat16*>(sb + off) = x;
  }
  tc::fence_proxy_async();
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  if (tid < 32) tc::tmem_alloc(&tmem_base, 128);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  if (tid == 0) {
    const uint32_t idesc = tc::idesc_bf16(M, N, a_mn, b_mn);
    const uint32_t a0 = tc::smem_u32(sa), b0 = tc::smem_u32(sb);
    for (int k0 = 0; k0 < K; k0 += 16) {
      const uint64_t ad = a_mn ? tc::desc_mnmajor_sw128(a0 + k0 * 128, K * 128)
                               : tc::desc_kmajor_sw128(a0 + (k0 >> 6) * M * 128 + (k0 & 63) * 2);
      const uint64_t bd = b_mn ? tc::desc_mnmajor_sw128(b0 + k0 * 128, K * 128)
                               : tc::desc_kmajor_sw128(b0 + (k0 >> 6) * N * 128 + (k0 & 63) * 2);
      tc::mma_bf16(tbase, ad, bd, idesc, k0 > 0);
    }
    tc::mma_commit(&bar);
  }
  tc::mbar_wait(&bar, 0, err, 1);
  tc::fence_after_sync();
  const int w = tid >> 5, l = tid & 31;
  for (int n0 = 0; n0 < N; n0 += 32) {
    float v[32];
    tc::tmem_ld32(tbase + (uint32_t(w * 32) << 16) + n0, v);
    int m;
    if (M == 128) m = w * 32 + l;
    else m = (l < 16) ? w * 16 + l : -1;  // M = 64: rows in lanes 0-15 of each 32-lane quarter
    if (m >= 0) {
      for (int j = 0; j < 32; ++j) D[m * N + n0 + j] = v[j];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (tid < 32) tc::tmem_dealloc(tbase, 128);
}

// The bounded wait that every kernel's mbarrier waits use, made to run out on purpose: a barrier that
// one arrival completes must be seen complete (else code 902 is recorded), and a barrier that nothing
// arrives on must give up after max_polls polls and record 901, after which the kernel returns.
__global__ void selftest_wait_kernel(int* __restrict__ status, uint32_t max_polls) {
  __shared__ uint64_t bar[2];
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar[0], 1);
    tc::mbar_init(&bar[1], 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(&bar[1])) : "memory");
    tc::mbar_wait_polls(&bar[1], 0, status, 902, max_polls);  // phase 0 of bar[1] has completed
    tc::mbar_wait_polls(&bar[0], 0, status, 901, max_polls);  // nothing completes phase 0 of bar[0]
  }
}

}  // namespace
}  // namespace rb2

extern "C" RB2_API int rb2_selftest_wait(int* status, unsigned int max_polls, void* stream) {
  using namespace rb2;
  RB2_CHECK_ARG(status && max_polls > 0 && max_polls <= (1u << 24), "selftest_wait: status and 0 < max_polls <= 2^24");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  selftest_wait_kernel<<<1, 32, 0, s>>>(status, max_polls);
  RB2_CHECK_LAUNCH("selftest_wait");
  return RB2_OK;
}

extern "C" RB2_API int rb2_selftest_mma(const void* A, const void* B, float* D, int a_mn, int b_mn, int M, int N,
                                        int K, int* err, void* stream) {
  using namespace rb2;
  RB2_CHECK_ARG((M == 64 || M == 128) && (N == 64 || N == 128) && (K == 64 || K == 128), "selftest_mma: shape");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t smem = 65536 + 1024;
  RB2_CUDA(cudaFuncSetAttribute(selftest_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
           "selftest_mma: smem attribute");
  selftest_mma_kernel<<<1, 128, smem, s>>>(static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(B),
                                           D, a_mn, b_mn, M, N, K, err);
  RB2_CHECK_LAUNCH("selftest_mma");
  return RB2_OK;
}
