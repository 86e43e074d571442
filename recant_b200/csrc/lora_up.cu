// LoRA up-projection added to a base output on tcgen05: out = y + s (h B^T), rounded as the
// reference's ops round it.
//
// The LoRA term of the GDN block's projections (recant/model/layers.py:65-70, 86-97) is
// y + (alpha / r) (h B^T) with h = x A^T [M, r] and B [N, r], r <= 128. torch runs it as one
// addmm (grouped_linear's default, layers.py:86-97: mode 0) or as three bf16 ops (QLinear.forward,
// layers.py:65-70: mode 1), which for out_proj read and write [M, N] bf16 tensors five times. Here
// one pass reads y, writes out, and the K = r product runs on the tensor core. The same pass also
// adds a narrow product to another output: the block's input gradient, dx + dproj [W_b; W_a; A]
// (r = 96), with mode 1 and s = 1.
//
//   mode 0: out = bf16(y + bf16(s * acc))                 (torch.addmm on the GPU: cuBLAS rounds the
//                                                          scaled product to bf16 before adding y)
//   mode 1: out = bf16(y + bf16(bf16(acc) * s))           (h B^T, * s, + y: three roundings)
// with acc = sum_k h[m, k] B[n, k] in fp32. Both are bit-identical to the reference's ops run by
// torch on a B200 (tests/test_lora_wgrad_gpu.py compares every element).
//
// One CTA (128 threads) per 128 x 128 output tile, three CTAs per SM for r <= 64, two above. Thread
// 0 loads the tile's h rows and B rows (one 64-column box each per 64 of r, columns past r
// zero-filled by TMA; 128-byte swizzle, no multicast) and, on a second barrier, y's tile (two
// 64-column boxes); it issues ceil(r / 16) tcgen05.mma (M = N = 128, K = 16, both operands K-major)
// as soon as h and B are in. Each thread
// then takes one output row: its accumulator columns from TMEM, y from the swizzled tile, the
// result written back over y in shared memory, and the tile leaves by two TMA stores (rows and
// columns past the tensor are clipped by TMA). Every mbarrier wait is bounded; a wait that runs out
// writes its code to the status word (the first 4 bytes of the workspace) and the kernel finishes.
#include "tmap.cuh"

namespace rb2 {
namespace {

constexpr int kTile = 128;
constexpr int kSlab = kTile * 128;            // 128 rows x 64 bf16: one SW128 slab of h, of B or of y
constexpr int kYBytes = 2 * kSlab;            // y / out tile: two 64-column slabs
constexpr int kMaxRank = 128;                 // h and B: one slab per 64 of r
inline int smem_bytes(int nslab) { return 2 * nslab * kSlab + kYBytes + 1024; }
constexpr size_t kStatusBytes = 256;

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(tc::smem_u32(smem_dst)),
      "l"(map), "r"(x), "r"(y), "r"(tc::smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(tc::smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}

// bf16 [rows][cols] with row stride ld elements, box 64 columns x 128 rows, 128-byte swizzle
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld) {
  auto fn = tmap_encoder();
  if (!fn) {
    set_error("lora_up: cuTensorMapEncodeTiled unavailable");
    return RB2_ECUDA;
  }
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {64u, cuuint32_t(kTile)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("lora_up: cuTensorMapEncodeTiled failed (%d)", int(r));
    return RB2_ECUDA;
  }
  return RB2_OK;
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(128, 2)
lora_up_kernel(const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_b,
               const __grid_constant__ CUtensorMap map_y, const __grid_constant__ CUtensorMap map_out, int r,
               int n_tiles_n, float s, int mode, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024 - (tc::smem_u32(smem_raw) & 1023)) & 1023);
  const int nslab = (r + 63) / 64;
  unsigned char* th = sm;
  unsigned char* tb = sm + nslab * kSlab;
  unsigned char* ty = tb + nslab * kSlab;
  __shared__ uint64_t bar_hb, bar_y, bar_mma;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int m0 = (int(blockIdx.x) / n_tiles_n) * kTile, n0 = (int(blockIdx.x) % n_tiles_n) * kTile;

  if (w == 0) {
    tc::tmem_alloc(&tmem_base, kTile);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&bar_hb, 1);
    tc::mbar_init(&bar_y, 1);
    tc::mbar_init(&bar_mma, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  bool ok = true;
  if (tid == 0) {
    tc::mbar_expect_tx(&bar_hb, uint32_t(2 * nslab * kSlab));
    for (int j = 0; j < nslab; ++j) {
      tma_load_2d(th + j * kSlab, &map_h, 64 * j, m0, &bar_hb);
      tma_load_2d(tb + j * kSlab, &map_b, 64 * j, n0, &bar_hb);
    }
    tc::mbar_expect_tx(&bar_y, uint32_t(kYBytes));
    tma_load_2d(ty, &map_y, n0, m0, &bar_y);
    tma_load_2d(ty + kYBytes / 2, &map_y, n0 + 64, m0, &bar_y);
    ok = tc::mbar_wait(&bar_hb, 0, err, 501);
    tc::fence_after_sync();
    if (ok) {
      constexpr uint32_t idesc = tc::idesc_bf16(kTile, kTile, false, false);
      const uint32_t sa = tc::smem_u32(th), sb = tc::smem_u32(tb);
      for (int k = 0; k * 16 < r; ++k) {  // 16 k = 32 bytes along a swizzled row; 64 k per slab
        const uint32_t off = uint32_t((k >> 2) * kSlab + (k & 3) * 32);
        tc::mma_bf16(tbase, tc::desc_kmajor_sw128(sa + off), tc::desc_kmajor_sw128(sb + off), idesc, k > 0);
      }
    }
    tc::mma_commit(&bar_mma);
  }
  __syncwarp();
  ok = tc::mbar_wait(&bar_mma, 0, err, 502) && tc::mbar_wait(&bar_y, 0, err, 503);
  tc::fence_after_sync();
  // thread (w, l): output row 32 w + l of the tile (TMEM lane), 32 columns at a time
  const int row = 32 * w + l;
#pragma unroll 1
  for (int c = 0; c < kTile / 32; ++c) {
    float acc[32];
    tc::tmem_ld32(tbase + (uint32_t(32 * w) << 16) + uint32_t(32 * c), acc);
    if (!ok) continue;
    unsigned char* slab = ty + (c >> 1) * (kYBytes / 2) + row * 128;
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // four 16-byte chunks of 8 columns
      const int chunk = (((c & 1) * 4 + q) ^ (row & 7));
      uint4* p = reinterpret_cast<uint4*>(slab + chunk * 16);
      const uint4 yv = *p;
      const uint32_t yw[4] = {yv.x, yv.y, yv.z, yv.w};
      uint32_t ow[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float y0 = __uint_as_float(yw[j] << 16), y1 = __uint_as_float(yw[j] & 0xffff0000u);
        const float a0 = acc[8 * q + 2 * j], a1 = acc[8 * q + 2 * j + 1];
        float o0, o1;
        if (mode == 0) {
          o0 = y0 + bf16r(s * a0);
          o1 = y1 + bf16r(s * a1);
        } else {
          o0 = y0 + bf16r(bf16r(a0) * s);
          o1 = y1 + bf16r(bf16r(a1) * s);
        }
        ow[j] = tc::pack_bf16(o0, o1);
      }
      *p = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
  }
  tc::fence_proxy_async();  // the generic-proxy writes of the tile, visible to the TMA store
  tc::fence_before_sync();
  __syncthreads();
  if (tid == 0) {
    if (ok) {
      tma_store_2d(&map_out, ty, n0, m0);
      tma_store_2d(&map_out, ty + kYBytes / 2, n0 + 64, m0);
      tc::bulk_commit();
    }
    tc::bulk_wait_all();  // the stores have left shared memory (and completed) before the CTA exits
  }
  __syncthreads();
  if (w == 0) tc::tmem_dealloc(tbase, kTile);
}

}  // namespace
}  // namespace rb2

using namespace rb2;

extern "C" size_t rb2_lora_up_workspace_size(void) { return kStatusBytes; }

extern "C" int rb2_lora_up(const void* y, int64_t ldy, const void* h, int64_t ldh, const void* b, int64_t ldb,
                           int64_t M, int64_t N, int r, float scale, int mode, void* out, int64_t ldo, void* ws,
                           size_t ws_bytes, void* stream) {
  RB2_CHECK_ARG(ws, "lora_up: null workspace");
  RB2_CHECK_ARG(M >= 0 && M < (int64_t(1) << 31) && N > 0 && N < (int64_t(1) << 31),
                "lora_up: need 0 <= M < 2^31 and 0 < N < 2^31 (M=%lld N=%lld)", (long long)M, (long long)N);
  RB2_CHECK_ARG(r >= 1 && r <= kMaxRank, "lora_up: rank must be in [1, 128] (r=%d)", r);
  RB2_CHECK_ARG(mode == 0 || mode == 1, "lora_up: mode must be 0 (addmm) or 1 (three ops)");
  RB2_CHECK_ARG(ws_bytes >= kStatusBytes && (reinterpret_cast<uintptr_t>(ws) & 15) == 0,
                "lora_up: workspace of at least %zu bytes, 16-byte aligned", kStatusBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* err = static_cast<int*>(ws);
  RB2_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s), "lora_up: clear status");
  if (M == 0) return RB2_OK;
  RB2_CHECK_ARG(y && h && b && out, "lora_up: null pointer");
  RB2_CHECK_ARG(ldy >= N && ldo >= N && ldh >= r && ldb >= r && ldy % 8 == 0 && ldo % 8 == 0 && ldh % 8 == 0 &&
                    ldb % 8 == 0,
                "lora_up: row strides must cover the rows and be multiples of 8 elements");
  RB2_CHECK_ARG(((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(b) |
                  reinterpret_cast<uintptr_t>(out)) & 15) == 0,
                "lora_up: y, h, B and out must be 16-byte aligned");
  CUtensorMap mh, mb, my, mo;
  int rc;
  if ((rc = make_map(&mh, h, M, r, ldh)) || (rc = make_map(&mb, b, N, r, ldb)) || (rc = make_map(&my, y, M, N, ldy)) ||
      (rc = make_map(&mo, out, M, N, ldo)))
    return rc;
  const int64_t tn = (N + kTile - 1) / kTile, tm = (M + kTile - 1) / kTile;
  RB2_CHECK_ARG(tn * tm < (int64_t(1) << 31), "lora_up: too many tiles");
  const int smem = smem_bytes((r + 63) / 64);
  cudaError_t e = cudaFuncSetAttribute(lora_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(2));
  if (e != cudaSuccess) {
    set_error("lora_up: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return RB2_ECUDA;
  }
  {
    ProfScope ps_("lora_up", s);
    lora_up_kernel<<<unsigned(tn * tm), 128, smem, s>>>(mh, mb, my, mo, r, int(tn), scale, mode, err);
  }
  RB2_CHECK_LAUNCH("lora_up");
  return RB2_OK;
}
