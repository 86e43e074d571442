// Narrow bf16 projections on tcgen05: out[M, N] = A[M, K] . B[N, K]^T with N <= 256.
//
// The GDN block's dense projections from the hidden state that are too narrow for NVFP4: the beta
// and gate projections in_proj_b / in_proj_a (recant/model/layers.py:154-155; N = Hv each, never
// quantized because N < 256, layers.py:47-48) and the LoRA down-projections x A^T of the quantized
// projections (layers.py:65-69, 86-88), all reading the same x. Concatenating their weights along
// N makes one pass over x produce all of them (N = 2 Hv + the LoRA ranks, 96 at the 9B shape).
//
// The product is bound by reading A (M x K bf16; B is at most 256 x K and stays in L2). One CTA per
// 128 rows of A, 128 threads: thread 0 streams A and B in 64-column (128-byte) slabs by TMA (128-byte
// swizzle, no multicast) through a 4-stage ring; thread 32 issues one tcgen05.mma (M = 128, N, K =
// 16) per 16 columns into an fp32 TMEM accumulator; then all four warps drain their 32 TMEM lanes
// (one output row per thread) and store bf16 or fp32. Rows of A past M read as zero (TMA fill) and
// are not stored. Every mbarrier wait is bounded.
#include "tmap.cuh"

namespace rb2 {
namespace {

constexpr int kRows = 128, kSlab = 64, kStages = 4;  // rows per CTA, K elements per stage

// A wait that runs out records its code here (the kernel then finishes without hanging)
__device__ int g_skinny_err;

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(tc::smem_u32(smem_dst)),
      "l"(map), "r"(x), "r"(y), "r"(tc::smem_u32(bar))
      : "memory");
}

// 2-D bf16 tensor [rows][cols] with row stride ld elements, box [box_rows][64 elements], 128-byte swizzle
int make_map_bf16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  auto fn = tmap_encoder();
  if (!fn) {
    set_error("skinny_gemm: cuTensorMapEncodeTiled unavailable");
    return RB2_ECUDA;
  }
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {cuuint32_t(kSlab), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("skinny_gemm: cuTensorMapEncodeTiled failed (%d)", int(r));
    return RB2_ECUDA;
  }
  return RB2_OK;
}

__global__ void __launch_bounds__(128, 1)
skinny_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, int M, int N,
                   int K, int tmem_cols, void* __restrict__ out, int64_t ldo, int out_bf16) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024 - (tc::smem_u32(smem_raw) & 1023)) & 1023);
  const int a_bytes = kRows * 128, b_bytes = N * 128, stage_bytes = a_bytes + ((b_bytes + 1023) & ~1023);
  __shared__ uint64_t full[kStages], empty[kStages], done;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int m0 = blockIdx.x * kRows, nk = K / kSlab;

  if (w == 0) {
    tc::tmem_alloc(&tmem_base, uint32_t(tmem_cols));
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(&done, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  if (tid == 0) {  // producer
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % kStages;
      if (!tc::mbar_wait(&empty[s], ((kt / kStages) & 1) ^ 1, &g_skinny_err, 301)) break;
      unsigned char* st = sm + s * stage_bytes;
      tc::mbar_expect_tx(&full[s], uint32_t(a_bytes + b_bytes));
      tma_load_2d(st, &map_a, kt * kSlab, m0, &full[s]);
      tma_load_2d(st + a_bytes, &map_b, kt * kSlab, 0, &full[s]);
    }
  } else if (tid == 32) {  // MMA issuer
    const uint32_t idesc = tc::idesc_bf16(kRows, N, false, false);
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % kStages;
      if (!tc::mbar_wait(&full[s], (kt / kStages) & 1, &g_skinny_err, 302)) break;
      tc::fence_after_sync();
      const uint32_t sa = tc::smem_u32(sm + s * stage_bytes), sb = sa + uint32_t(a_bytes);
#pragma unroll
      for (int kk = 0; kk < kSlab / 16; ++kk)
        tc::mma_bf16(tbase, tc::desc_kmajor_sw128(sa + 32 * kk), tc::desc_kmajor_sw128(sb + 32 * kk), idesc,
                     kt > 0 || kk > 0);
      tc::mma_commit(&empty[s]);
    }
    tc::mma_commit(&done);
  }
  __syncwarp();
  tc::mbar_wait(&done, 0, &g_skinny_err, 303);
  tc::fence_after_sync();
  // warp w drains TMEM lanes 32 w .. 32 w + 31: output row m0 + 32 w + l, 16 columns at a time
  const int row = m0 + 32 * w + l;
  for (int c = 0; c < N; c += 16) {
    float v[16];
    tc::tmem_ld16(tbase + (uint32_t(32 * w) << 16) + uint32_t(c), v);
    if (row < M) {
      if (out_bf16) {
        uint4* o = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + int64_t(row) * ldo + c);
        o[0] = make_uint4(tc::pack_bf16(v[0], v[1]), tc::pack_bf16(v[2], v[3]), tc::pack_bf16(v[4], v[5]),
                          tc::pack_bf16(v[6], v[7]));
        o[1] = make_uint4(tc::pack_bf16(v[8], v[9]), tc::pack_bf16(v[10], v[11]), tc::pack_bf16(v[12], v[13]),
                          tc::pack_bf16(v[14], v[15]));
      } else {
        float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + int64_t(row) * ldo + c);
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (w == 0) tc::tmem_dealloc(tbase, uint32_t(tmem_cols));
}

}  // namespace
}  // namespace rb2

using namespace rb2;

extern "C" int rb2_skinny_gemm(const void* a, int64_t lda, const void* b, int64_t M, int64_t N, int64_t K, void* out,
                               int64_t ldo, int out_dtype, void* stream) {
  RB2_CHECK_ARG(a && b && out, "skinny_gemm: null pointer");
  RB2_CHECK_ARG(M > 0 && M < (int64_t(1) << 31) && K > 0 && K % 64 == 0 && K < (int64_t(1) << 31),
                "skinny_gemm: need M > 0 and K a positive multiple of 64 (M=%lld K=%lld)", (long long)M, (long long)K);
  RB2_CHECK_ARG(N >= 16 && N <= 256 && N % 16 == 0, "skinny_gemm: N must be a multiple of 16 in [16, 256] (N=%lld)",
                (long long)N);
  RB2_CHECK_ARG(out_dtype == RB2_F32 || out_dtype == RB2_BF16, "skinny_gemm: out_dtype");
  RB2_CHECK_ARG(lda >= K && lda % 8 == 0 && ldo >= N && ldo % 8 == 0,
                "skinny_gemm: row strides must cover the rows and be multiples of 8 elements (lda=%lld ldo=%lld)",
                (long long)lda, (long long)ldo);
  RB2_CHECK_ARG((reinterpret_cast<uintptr_t>(a) & 15) == 0 && (reinterpret_cast<uintptr_t>(b) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(out) & 15) == 0,
                "skinny_gemm: A, B and out must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int b_pad = (int(N) * 128 + 1023) & ~1023;
  const int smem = kStages * (kRows * 128 + b_pad) + 1024;
  int tmem_cols = 32;
  while (tmem_cols < N) tmem_cols <<= 1;
  // the first CUDA call also makes the device's context current on a thread that has not used it yet,
  // which the tensor-map encoding below needs
  cudaError_t e = cudaFuncSetAttribute(skinny_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    set_error("skinny_gemm: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return RB2_ECUDA;
  }
  CUtensorMap ma, mb;
  int rc;
  if ((rc = make_map_bf16(&ma, a, M, K, lda, kRows)) || (rc = make_map_bf16(&mb, b, N, K, K, int(N)))) return rc;
  {
    ProfScope ps_("skinny_gemm", s);
    skinny_gemm_kernel<<<unsigned((M + kRows - 1) / kRows), 128, smem, s>>>(ma, mb, int(M), int(N), int(K), tmem_cols,
                                                                          out, ldo, out_dtype == RB2_BF16);
  }
  RB2_CHECK_LAUNCH("skinny_gemm");
  return RB2_OK;
}

extern "C" int rb2_skinny_gemm_status(int* code, int clear) {
  RB2_CHECK_ARG(code, "skinny_gemm_status: null pointer");
  RB2_CUDA(cudaDeviceSynchronize(), "skinny_gemm_status: synchronize");
  RB2_CUDA(cudaMemcpyFromSymbol(code, g_skinny_err, sizeof(int)), "skinny_gemm_status: read");
  if (clear) {
    const int zero = 0;
    RB2_CUDA(cudaMemcpyToSymbol(g_skinny_err, &zero, sizeof(int)), "skinny_gemm_status: clear");
  }
  return RB2_OK;
}
