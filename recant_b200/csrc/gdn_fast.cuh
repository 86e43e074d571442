// Shared declarations of the tensor-core GDN path (gdn_fast.cu forward, gdn_fast_bwd.cu backward).
#pragma once

#include "gdn_common.cuh"
#include "tc.cuh"

namespace rb2 {

struct FastWs {
  ChunkTable ct;
  float* stats;          // [ch][8][64] cum, rq, rk, beta, f_q = scale rq e^cum, f_k = rk e^(cl - cum), e^cum, e^(cl - cum)
  __nv_bfloat16* tinv;   // [ch][64][64]   T = (I + L)^-1                      (tile image)
  __nv_bfloat16* aqk;    // [ch][64][64]   (q k^T) Gamma * scales, lower incl. diagonal (image)
  __nv_bfloat16* w;      // [ch][64][128]                                      (tile image)
  __nv_bfloat16* u;      // [ch][64][128]   plain row-major
  __nv_bfloat16* qt;     // [ch][64][128]  q~ = f_q q, for the backward walk (tile image)
  __nv_bfloat16* hs;     // [ch][128][128] S^T entering the chunk, [dv][dk] (tile image)
  __nv_bfloat16* vp;     // [ch][128][64]  V'^T [dv][tok] (tile image)
  __nv_bfloat16* dh;     // [ch][128][128] dS^T of the state leaving the chunk, [dv][dk] (image)
  __nv_bfloat16* dvp;    // [ch][128][64]  dV'^T [dv][tok] (tile image)
  int* err;              // device status word
};

// The workspace has two parts: "saved" (written by the forward, read by the backward: chunk table,
// status word, per-chunk prep outputs, states and V') and "scratch" (backward only: dS and dV'),
// which the caller may pass separately and reuse across layers.
size_t carve_fast_saved(Carver& c, FastWs& w, int64_t n_seqs, int Hv, int max_chunks);
size_t carve_fast_scratch(Carver& c, FastWs& w, int64_t tokens, int Hv, int max_chunks, bool gqa);

namespace fast {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ unsigned char* align1024(unsigned char* p) {
  return p + ((1024 - (tc::smem_u32(p) & 1023)) & 1023);
}

// Asynchronously copy `nrows` rows of 128 bf16 (row stride `stride` elements) into rows
// [r0, r0+nrows) of a K-major SW128 tile with `tile_rows` rows; rows >= L are zero-filled. All
// `nthr` threads participate; completion via cp_async_commit / cp_async_wait.
__device__ __forceinline__ void load_rows_sw128(unsigned char* tile, int tile_rows, int r0, const bf16* src,
                                                int64_t stride, int nrows, int L, int nthr) {
  for (int idx = threadIdx.x; idx < nrows * 16; idx += nthr) {
    const int r = idx >> 4, c8 = idx & 15;
    const bool ok = r < L;
    tc::cp_async16(tile + tc::sw128_offset(r0 + r, c8 * 8, tile_rows), src + (ok ? r * stride + c8 * 8 : 0), ok);
  }
}

// Rows of 64 bf16 (e.g. a 64x64 A_qk block, row stride 64) into a one-slab SW128 tile.
__device__ __forceinline__ void load_rows64_sw128(unsigned char* tile, const bf16* src, int nthr) {
  for (int idx = threadIdx.x; idx < 64 * 8; idx += nthr) {
    const int i = idx >> 3, c8 = idx & 7;
    tc::cp_async16(tile + tc::sw128_offset(i, c8 * 8, 64), src + i * 64 + c8 * 8, true);
  }
}

// Same for a plain row-major [64][128] bf16 smem tile (no swizzle).
__device__ __forceinline__ void load_rows_plain(bf16* tile, const bf16* src, int64_t stride, int nthr) {
  for (int idx = threadIdx.x; idx < 64 * 16; idx += nthr) {
    const int r = idx >> 4, c8 = idx & 15;
    tc::cp_async16(tile + r * 128 + c8 * 8, src + r * stride + c8 * 8, true);
  }
}

__device__ __forceinline__ float bf_lo(uint32_t x) { return __uint_as_float(x << 16); }
// N consecutive floats of a per-token vector in shared memory (16-byte aligned) by 16-byte loads
template <int N>
__device__ __forceinline__ void lds_vec(const float* p, float (&out)[N]) {
#pragma unroll
  for (int k = 0; k < N; k += 4) *reinterpret_cast<float4*>(out + k) = *reinterpret_cast<const float4*>(p + k);
}
constexpr float kLog2e = 1.4426950408889634f;  // log2(e)
// 2^x by the hardware approximation (MUFU.EX2; denormal results flush to zero)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float bf_hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }

// (I + L)^-1 for strictly-lower L (fp32 64x64, stride 65) into T (stride 65); `nthr` threads, a
// multiple of 128 and at least 256. The four 16x16 diagonal blocks by forward substitution (warps
// 0-3, lane = column) while warps 4-7 zero the blocks above the diagonal; then the off-diagonal blocks by block
// rows, T_ij = -T_ii X_j with X_j = sum_{j<=m<i} L_im T_mj. Each thread of a block-row step owns a
// 2x2 tile of one X_j and then of T_ij (a warp: one j, 4 x 8 tiles), so that every shared-memory
// value it loads feeds two FMAs; every element is still one fma chain in ascending m.
__device__ inline void unit_lower_inverse(const float* lm, float* tm, float* xbuf, int nthr) {
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  if (w < 4) {
    if (l < 16) {  // warp w inverts diagonal block w by forward substitution, lane = column
      const int o = 16 * w;
      float col[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float t = (i == l) ? 1.f : 0.f;
#pragma unroll
        for (int m = 0; m < i; ++m) t = fmaf(-lm[(o + i) * 65 + o + m], col[m], t);
        col[i] = t;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) tm[(o + i) * 65 + o + l] = col[i];
    }
  } else {
    for (int idx = tid - 128; idx < 6 * 256; idx += nthr - 128) {  // the six blocks above the diagonal
      const int b = idx >> 8, bi = b < 3 ? 0 : (b < 5 ? 1 : 2), bj = b < 3 ? b + 1 : (b < 5 ? b - 1 : 3);
      tm[(16 * bi + ((idx >> 4) & 15)) * 65 + 16 * bj + (idx & 15)] = 0.f;
    }
  }
  __syncthreads();
  for (int bi = 1; bi < 4; ++bi) {
    for (int t = tid; t < 64 * bi; t += nthr) {  // X_bj rows 2 r2, 2 r2 + 1, columns 2 cc, 2 cc + 1
      const int bj = t >> 6, r2 = (t >> 3) & 7, cc = t & 7;
      const float* a = lm + (16 * bi + 2 * r2) * 65;
      const float* b = tm + 16 * bj + 2 * cc;
      float x00 = 0.f, x01 = 0.f, x10 = 0.f, x11 = 0.f;
      for (int m = 16 * bj; m < 16 * bi; ++m) {
        const float a0 = a[m], a1 = a[65 + m], b0 = b[m * 65], b1 = b[m * 65 + 1];
        x00 = fmaf(a0, b0, x00);
        x01 = fmaf(a0, b1, x01);
        x10 = fmaf(a1, b0, x10);
        x11 = fmaf(a1, b1, x11);
      }
      float* xo = xbuf + bj * 256 + 2 * r2 * 16 + 2 * cc;
      *reinterpret_cast<float2*>(xo) = make_float2(x00, x01);
      *reinterpret_cast<float2*>(xo + 16) = make_float2(x10, x11);
    }
    __syncthreads();
    for (int t = tid; t < 64 * bi; t += nthr) {  // T_bi,bj = -T_bi,bi X_bj, same tiles
      const int bj = t >> 6, r2 = (t >> 3) & 7, cc = t & 7;
      const float* a = tm + (16 * bi + 2 * r2) * 65 + 16 * bi;
      const float* xb = xbuf + bj * 256 + 2 * cc;
      float t00 = 0.f, t01 = 0.f, t10 = 0.f, t11 = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float a0 = a[m], a1 = a[65 + m];
        const float2 x = *reinterpret_cast<const float2*>(xb + m * 16);
        t00 = fmaf(a0, x.x, t00);
        t01 = fmaf(a0, x.y, t01);
        t10 = fmaf(a1, x.x, t10);
        t11 = fmaf(a1, x.y, t11);
      }
      float* to = tm + (16 * bi + 2 * r2) * 65 + 16 * bj + 2 * cc;
      to[0] = -t00;
      to[1] = -t01;
      to[65] = -t10;
      to[66] = -t11;
    }
    __syncthreads();
  }
}

// 32 bf16 (64 bytes) of row r starting at element e0 of a K-major SW128 tile -> fp32
__device__ __forceinline__ void store_row32(unsigned char* tile, int rows, int r, int e0, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 x = make_uint4(tc::pack_bf16(v[8 * j], v[8 * j + 1]), tc::pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                               tc::pack_bf16(v[8 * j + 4], v[8 * j + 5]), tc::pack_bf16(v[8 * j + 6], v[8 * j + 7]));
    *reinterpret_cast<uint4*>(tile + tc::sw128_offset(r, e0 + 8 * j, rows)) = x;
  }
}

// 16 values of row r starting at element e0 (a multiple of 8) of a K-major SW128 tile -> bf16
__device__ __forceinline__ void store_row16(unsigned char* tile, int rows, int r, int e0, const float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const uint4 x = make_uint4(tc::pack_bf16(v[8 * j], v[8 * j + 1]), tc::pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                               tc::pack_bf16(v[8 * j + 4], v[8 * j + 5]), tc::pack_bf16(v[8 * j + 6], v[8 * j + 7]));
    *reinterpret_cast<uint4*>(tile + tc::sw128_offset(r, e0 + 8 * j, rows)) = x;
  }
}

// 8 values of row r starting at element e0 (a multiple of 8) of a K-major SW128 tile -> bf16
__device__ __forceinline__ void store_row8(unsigned char* tile, int rows, int r, int e0, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(tile + tc::sw128_offset(r, e0, rows)) =
      make_uint4(tc::pack_bf16(v[0], v[1]), tc::pack_bf16(v[2], v[3]), tc::pack_bf16(v[4], v[5]), tc::pack_bf16(v[6], v[7]));
}

// store_cols32 for 16 tokens (t_base + j, j < 16)
__device__ __forceinline__ void store_cols16(bf16* dst, int row, int r, int t_base, int L, const float (&v)[16]) {
  const bool odd = (r & 1) != 0;
  const int t_odd = t_base + (odd ? 1 : 0);
  uint32_t* base = reinterpret_cast<uint32_t*>(dst + t_odd * row + (r & ~1));
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    const float other = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
    const float lo = odd ? other : v[j], hi = odd ? v[j + 1] : other;
    if (t_odd + j < L) base[(j * row) >> 1] = tc::pack_bf16(lo, hi);
  }
}

// Write 32 per-token values of head-dim column r (tokens 32 hh + j) as bf16 to dst[(tok) * row + r],
// pairing lanes r, r^1 so that every store is one 4-byte bf16x2.
// `row` elements between tokens; the 64 tokens of a chunk span less than 2^31 elements.
__device__ __forceinline__ void store_cols32(bf16* dst, int row, int r, int t_base, int L, const float (&v)[32]) {
  const bool odd = (r & 1) != 0;
  const int t_odd = t_base + (odd ? 1 : 0);
  uint32_t* base = reinterpret_cast<uint32_t*>(dst + t_odd * row + (r & ~1));
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float other = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
    const float lo = odd ? other : v[j], hi = odd ? v[j + 1] : other;
    if (t_odd + j < L) base[(j * row) >> 1] = tc::pack_bf16(lo, hi);
  }
}

// Workspace tiles that a later kernel loads as an MMA operand are stored as "images": the exact
// bytes of the K-major SW128 shared-memory tile (tc::sw128_offset), so that one linear bulk copy
// into a 1024-byte-aligned buffer reproduces the swizzled operand.
__device__ __forceinline__ unsigned char* img(void* base) { return static_cast<unsigned char*>(base); }

// 32 per-token values of head-dim column r (tokens t_base + j) into a plain [64][128] tile in shared
// memory: bf16 pairs from lanes r, r^1, or fp32 words
__device__ __forceinline__ void stage_cols32(bf16* tile, int r, int t_base, const float (&v)[32]) {
  const bool odd = (r & 1) != 0;
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float other = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
    const int tk = t_base + j + (odd ? 1 : 0);
    const float lo = odd ? other : v[j], hi = odd ? v[j + 1] : other;
    *reinterpret_cast<uint32_t*>(tile + tk * 128 + (r & ~1)) = tc::pack_bf16(lo, hi);
  }
}
__device__ __forceinline__ void stage_cols16(bf16* tile, int r, int t_base, const float (&v)[16]) {
  const bool odd = (r & 1) != 0;
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    const float other = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
    const int tk = t_base + j + (odd ? 1 : 0);
    const float lo = odd ? other : v[j], hi = odd ? v[j + 1] : other;
    *reinterpret_cast<uint32_t*>(tile + tk * 128 + (r & ~1)) = tc::pack_bf16(lo, hi);
  }
}
__device__ __forceinline__ void stage_cols32(float* tile, int r, int t_base, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) tile[(t_base + j) * 128 + r] = v[j];
}
// Rows [0, L) of a plain [64][row_elems] shared tile to dst + i * stride (16-byte chunks by nthr
// threads starting at thread `first`; row_bytes a multiple of 16)
__device__ __forceinline__ void copy_rows_out(void* dst, int64_t stride_bytes, const void* tile, int row_bytes, int L,
                                              int first, int nthr) {
  const int chunks = row_bytes / 16;
  for (int idx = int(threadIdx.x) - first; idx >= 0 && idx < 64 * chunks; idx += nthr) {
    const int i = idx / chunks, c = idx - i * chunks;
    if (i < L)
      *reinterpret_cast<uint4*>(static_cast<char*>(dst) + i * stride_bytes + c * 16) =
          *reinterpret_cast<const uint4*>(static_cast<const char*>(tile) + i * row_bytes + c * 16);
  }
}

// store_cols32 into a tile image with `rows` rows: token t_base + j, head-dim column r.
__device__ __forceinline__ void store_cols32_img(unsigned char* image, int rows, int r, int t_base,
                                                 const float (&v)[32]) {
  const bool odd = (r & 1) != 0;
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float other = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
    const int tk = t_base + j + (odd ? 1 : 0);
    const float lo = odd ? other : v[j], hi = odd ? v[j + 1] : other;
    *reinterpret_cast<uint32_t*>(image + tc::sw128_offset(tk, r & ~1, rows)) = tc::pack_bf16(lo, hi);
  }
}

}  // namespace fast
}  // namespace rb2
