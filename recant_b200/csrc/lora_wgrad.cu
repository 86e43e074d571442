// LoRA weight gradients on tcgen05: out(n, r) = s * sum_m D[m, n] H[m, r], reduced over tokens m.
//
// The trainable parameters of the GDN block are its LoRA factors (recant/model/layers.py:55-60,
// 65-70, 86-97), and their gradients are products of this shape, reduced over all B*T tokens:
//   dB = s dy^T h      (D = dy [M, out], H = h = x A^T [M, r]; autograd of addmm / mm * s)
//   dA = (x^T dh)^T    (D = x [M, in],   H = dh [M, r];       autograd of x A^T)
// with r <= 64. Each is bound by reading D once (M x N bf16); H is M x r and mostly comes from L2.
//
// One CTA (128 threads) per (256 columns of D, split of the tokens), one CTA per SM. Thread 0 streams
// 64-token stages by TMA (four 64 x 64 boxes of D -- 512-byte runs of each row, which the DRAM
// pages serve better than 256-byte ones -- and one 64 x 64 box of H; 128-byte swizzle, no multicast)
// through a 4-stage ring; thread 32 issues, per stage and per 128-column half, four tcgen05.mma
// (M = 128 columns n, N = 64 columns r, K = 16 tokens) with both operands MN-major -- the tiles
// land token-major, as D and H are stored, and are read transposed by the descriptors, so nothing
// is transposed in memory. The fp32 accumulators (TMEM lanes = n, 64 columns per half) go to a
// per-split partial in the workspace; the last split of a column tile to arrive (an atomic counter
// per tile) sums the tile's partials in split order (deterministic) and rounds as the reference
// does: the bf16 product, then times s in bf16, stored as fp32 (the fp32 parameter's gradient
// through its bf16 cast, layers.py:69, 86, 95). The splits fill at most one wave. Columns of H
// past r, and tokens past M, read as zero (TMA fill). Every mbarrier wait is bounded; a wait that
// runs out writes its code to the status word (the first 4 bytes of the workspace) and the kernel
// finishes.
#include "tmap.cuh"

namespace rb2 {
namespace {

constexpr int kTok = 64;                      // tokens per stage
constexpr int kStages = 4;
constexpr int kHalves = 2;                    // 128-column halves of a tile: 256 columns of D per CTA
constexpr int kTileN = 128 * kHalves;
constexpr int kDBytes = kHalves * 2 * 64 * 128;  // D: four 64-column slabs of 64 token rows
constexpr int kHBytes = 64 * 128;             // H: one 64-column slab
constexpr int kStageBytes = kDBytes + kHBytes;
constexpr int kSmem = kStages * kStageBytes + 1024;
constexpr int kCols = 64;                     // accumulator columns per half (r padded to 64)
constexpr size_t kStatusBytes = 256;
// token splits per column tile, at most: fewer, longer splits leave less for the last CTA of a tile
// to sum (measured at 16384 x 4096: r 16 41.3 -> 39.9 us, r 32 51.5 -> 47.9 us from 9 splits to 6;
// 4 splits: 42.5 / 49.4 us)
constexpr int kMaxSplits = 6;

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(tc::smem_u32(smem_dst)),
      "l"(map), "r"(x), "r"(y), "r"(tc::smem_u32(bar))
      : "memory");
}

// bf16 [rows][cols] with row stride ld elements, box 64 columns x 64 rows, 128-byte swizzle
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t ld) {
  auto fn = tmap_encoder();
  if (!fn) {
    set_error("lora_wgrad: cuTensorMapEncodeTiled unavailable");
    return RB2_ECUDA;
  }
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {64u, cuuint32_t(kTok)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("lora_wgrad: cuTensorMapEncodeTiled failed (%d)", int(r));
    return RB2_ECUDA;
  }
  return RB2_OK;
}

// The reference's rounding of one gradient element: bf16 product, times s in bf16, as fp32.
__device__ __forceinline__ float finish(float acc, float s) {
  const float p = __bfloat162float(__float2bfloat16_rn(acc));
  return __bfloat162float(__float2bfloat16_rn(p * s));
}

__global__ void __launch_bounds__(128, 1)
lora_wgrad_kernel(const __grid_constant__ CUtensorMap map_d, const __grid_constant__ CUtensorMap map_h, int M, int N,
                  int R, int tok_per_split, int n_tiles, int n_splits, float s, float* __restrict__ partial,
                  int* __restrict__ arrivals, float* __restrict__ out, int64_t ld_n, int64_t ld_r,
                  int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024 - (tc::smem_u32(smem_raw) & 1023)) & 1023);
  __shared__ uint64_t full[kStages], empty[kStages], done;
  __shared__ uint32_t tmem_base;
  __shared__ int last;
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int tile = int(blockIdx.x) % n_tiles, split = int(blockIdx.x) / n_tiles;
  const int n0 = tile * kTileN, m0 = split * tok_per_split;
  const int m1 = min(M, m0 + tok_per_split);
  const int nk = (m1 - m0 + kTok - 1) / kTok;  // >= 1: the host sizes the splits so that none is empty

  if (w == 0) {
    tc::tmem_alloc(&tmem_base, kCols * kHalves);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int st = 0; st < kStages; ++st) {
      tc::mbar_init(&full[st], 1);
      tc::mbar_init(&empty[st], 1);
    }
    tc::mbar_init(&done, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  if (tid == 0) {  // producer: a split's stages never cross into the next split (tok_per_split % 64 == 0)
    for (int kt = 0; kt < nk; ++kt) {
      const int st = kt % kStages;
      if (!tc::mbar_wait(&empty[st], ((kt / kStages) & 1) ^ 1, err, 401)) break;
      unsigned char* b = sm + st * kStageBytes;
      const int y = m0 + kt * kTok;
      tc::mbar_expect_tx(&full[st], uint32_t(kStageBytes));
#pragma unroll
      for (int j = 0; j < 2 * kHalves; ++j) tma_load_2d(b + j * 8192, &map_d, n0 + 64 * j, y, &full[st]);
      tma_load_2d(b + kDBytes, &map_h, 0, y, &full[st]);
    }
  } else if (tid == 32) {  // MMA issuer: C[n][r] += D^T H over 16 tokens per instruction
    constexpr uint32_t idesc = tc::idesc_bf16(128, kCols, true, true);
    for (int kt = 0; kt < nk; ++kt) {
      const int st = kt % kStages;
      if (!tc::mbar_wait(&full[st], (kt / kStages) & 1, err, 402)) break;
      tc::fence_after_sync();
      const uint32_t sa = tc::smem_u32(sm + st * kStageBytes), sb = sa + uint32_t(kDBytes);
      // MN-major operands: a half's two 64-column slabs of D are 8 KB apart (LBO); 16 tokens = 2 KB;
      // half hv accumulates in TMEM columns 64 hv ..
      const uint64_t db = tc::desc_mnmajor_sw128(sb, kHBytes);
#pragma unroll
      for (int hv = 0; hv < kHalves; ++hv) {
        const uint64_t da = tc::desc_mnmajor_sw128(sa + uint32_t(hv * 16384), 8192);
#pragma unroll
        for (int kk = 0; kk < kTok / 16; ++kk)
          tc::mma_bf16(tbase + uint32_t(kCols * hv), da + uint64_t(kk * 128), db + uint64_t(kk * 128), idesc,
                       kt > 0 || kk > 0);
      }
      tc::mma_commit(&empty[st]);
    }
    tc::mma_commit(&done);
  }
  __syncwarp();
  const bool ok = tc::mbar_wait(&done, 0, err, 403);
  tc::fence_after_sync();
  // warp w holds TMEM lanes 32 w .. 32 w + 31: column n0 + 128 hv + 32 w + l of D in half hv
  const int64_t npad = int64_t(n_tiles) * kTileN;
#pragma unroll
  for (int hv = 0; hv < kHalves; ++hv) {
    const int n = n0 + 128 * hv + 32 * w + l;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float v[32];
      tc::tmem_ld32(tbase + (uint32_t(32 * w) << 16) + uint32_t(kCols * hv + 32 * half), v);
      if (!ok) continue;
      if (partial) {
        float4* p = reinterpret_cast<float4*>(partial + (int64_t(split) * npad + n) * kCols + 32 * half);
#pragma unroll
        for (int j = 0; j < 8; ++j) p[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      } else if (n < N) {  // a single split: finish here
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int r = 32 * half + j;
          if (r < R) out[int64_t(n) * ld_n + int64_t(r) * ld_r] = finish(v[j], s);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (w == 0) tc::tmem_dealloc(tbase, kCols * kHalves);
  if (!partial) return;
  // The last split of this column tile to finish sums all splits' partials, in split order (so the
  // result does not depend on which CTA came last), and writes the tile's output columns.
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&arrivals[tile], 1) == n_splits - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int hv = 0; hv < kHalves; ++hv) {
    const int n = n0 + 128 * hv + 32 * w + l;
    if (n >= N) break;
    // all splits' partials of two 4-column groups in flight at once (independent loads), then summed
    // in split order: a serial load-add chain over the splits would add one L2 round trip per partial
    for (int r8 = 0; r8 < R; r8 += 8) {
      float4 v[2][kMaxSplits];
#pragma unroll
      for (int g = 0; g < 2; ++g)
#pragma unroll
        for (int sp = 0; sp < kMaxSplits; ++sp)
          if (sp < n_splits && r8 + 4 * g < R)
            v[g][sp] = __ldcg(reinterpret_cast<const float4*>(partial + (int64_t(sp) * npad + n) * kCols + r8 + 4 * g));
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int sp = 0; sp < kMaxSplits; ++sp)
          if (sp < n_splits) {
            acc.x += v[g][sp].x;
            acc.y += v[g][sp].y;
            acc.z += v[g][sp].z;
            acc.w += v[g][sp].w;
          }
        const float a[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = r8 + 4 * g + j;
          if (r < R) out[int64_t(n) * ld_n + int64_t(r) * ld_r] = finish(a[j], s);
        }
      }
    }
  }
}

// out(n, r) = finish(0): the gradient over an empty token range
__global__ void lora_wgrad_zero_kernel(int N, int R, float s, float* __restrict__ out, int64_t ld_n, int64_t ld_r) {
  const int64_t total = int64_t(N) * R;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int n = int(i / R), r = int(i - int64_t(n) * R);
    out[int64_t(n) * ld_n + int64_t(r) * ld_r] = finish(0.f, s);
  }
}

// Token splits: as many as fit in one wave of one CTA on each of B200's 148 SMs (a second, partial
// wave would nearly double the time of a bandwidth-bound pass), whole 64-token stages per split.
void plan(int64_t M, int64_t N, int* n_tiles, int* n_splits, int* tok_per_split) {
  *n_tiles = int((N + kTileN - 1) / kTileN);
  const int64_t stages = (M + kTok - 1) / kTok;
  int want = 148 / *n_tiles;
  if (want > kMaxSplits) want = kMaxSplits;
  if (want < 1) want = 1;
  if (want > stages) want = int(stages);
  const int64_t per = (stages + want - 1) / want;  // stages per split
  *tok_per_split = int(per * kTok);
  *n_splits = int((stages + per - 1) / per);
}

}  // namespace
}  // namespace rb2

using namespace rb2;

extern "C" size_t rb2_lora_wgrad_workspace_size(int64_t M, int64_t N, int R) {
  (void)R;
  if (M <= 0 || N <= 0) return kStatusBytes;
  int n_tiles, n_splits, tok;
  plan(M, N, &n_tiles, &n_splits, &tok);
  if (n_splits == 1) return kStatusBytes;
  const size_t counters = (size_t(n_tiles) * sizeof(int) + 255) & ~size_t(255);
  return kStatusBytes + counters + size_t(n_splits) * size_t(n_tiles) * kTileN * kCols * sizeof(float);
}

extern "C" int rb2_lora_wgrad(const void* D, int64_t ldd, const void* H, int64_t ldh, int64_t M, int64_t N, int R,
                              float scale, float* out, int64_t ld_n, int64_t ld_r, void* ws, size_t ws_bytes,
                              void* stream) {
  RB2_CHECK_ARG(out && ws && (M == 0 || (D && H)), "lora_wgrad: null pointer");
  RB2_CHECK_ARG(M >= 0 && M < (int64_t(1) << 31) && N > 0 && N < (int64_t(1) << 31),
                "lora_wgrad: need 0 <= M < 2^31 and 0 < N < 2^31 (M=%lld N=%lld)", (long long)M, (long long)N);
  RB2_CHECK_ARG(R >= 1 && R <= kCols, "lora_wgrad: rank must be in [1, 64] (R=%d)", R);
  RB2_CHECK_ARG(ldd >= N && ldd % 8 == 0 && ldh >= R && ldh % 8 == 0,
                "lora_wgrad: row strides must cover the rows and be multiples of 8 elements (ldd=%lld ldh=%lld)",
                (long long)ldd, (long long)ldh);
  RB2_CHECK_ARG((reinterpret_cast<uintptr_t>(D) & 15) == 0 && (reinterpret_cast<uintptr_t>(H) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(ws) & 255) == 0,
                "lora_wgrad: D and H must be 16-byte aligned, the workspace 256-byte aligned");
  const size_t need = rb2_lora_wgrad_workspace_size(M, N, R);
  RB2_CHECK_ARG(ws_bytes >= need, "lora_wgrad: workspace of %zu bytes, %zu needed", ws_bytes, need);
  RB2_CHECK_ARG((ld_r == 1 && ld_n >= R) || (ld_n == 1 && ld_r >= N),
                "lora_wgrad: out must be [N, R] (ld_r 1) or [R, N] (ld_n 1) with rows covering it");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* err = static_cast<int*>(ws);
  if (M == 0) {  // an empty token range: the gradient is zero
    RB2_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s), "lora_wgrad: clear status");
    const int64_t total = N * R;
    {
      ProfScope ps_("lora_wgrad_zero", s);
      lora_wgrad_zero_kernel<<<unsigned((total + 255) / 256 < 4 * 148 ? (total + 255) / 256 : 4 * 148), 256, 0, s>>>(
          int(N), R, scale, out, ld_n, ld_r);
    }
    RB2_CHECK_LAUNCH("lora_wgrad zero");
    return RB2_OK;
  }
  int n_tiles, n_splits, tok;
  plan(M, N, &n_tiles, &n_splits, &tok);
  // workspace: status word | the column tiles' arrival counters | per-split partials
  const size_t counters = (size_t(n_tiles) * sizeof(int) + 255) & ~size_t(255);
  int* arrivals = n_splits > 1 ? reinterpret_cast<int*>(static_cast<char*>(ws) + kStatusBytes) : nullptr;
  float* partial =
      n_splits > 1 ? reinterpret_cast<float*>(static_cast<char*>(ws) + kStatusBytes + counters) : nullptr;
  // one memset clears the status word and the counters; as the call's first CUDA call it also makes
  // the device's context current on a thread that has not used it yet (an autograd worker), which
  // the tensor-map encoding below needs
  RB2_CUDA(cudaMemsetAsync(ws, 0, n_splits > 1 ? kStatusBytes + counters : sizeof(int), s), "lora_wgrad: clear");
  CUtensorMap md, mh;
  int rc;
  if ((rc = make_map(&md, D, M, N, ldd)) || (rc = make_map(&mh, H, M, R, ldh))) return rc;
  cudaError_t e = cudaFuncSetAttribute(lora_wgrad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) {
    set_error("lora_wgrad: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return RB2_ECUDA;
  }
  {
    ProfScope ps_("lora_wgrad", s);
    lora_wgrad_kernel<<<unsigned(n_tiles * n_splits), 128, kSmem, s>>>(md, mh, int(M), int(N), R, tok, n_tiles,
                                                                      n_splits, scale, partial, arrivals, out, ld_n,
                                                                      ld_r, err);
  }
  RB2_CHECK_LAUNCH("lora_wgrad");
  return RB2_OK;
}
