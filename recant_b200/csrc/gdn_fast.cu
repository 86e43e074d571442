// Chunked Gated DeltaNet, tensor-core path (bf16 operands, fp32 accumulation and state) on tcgen05.
//
// Same chunked factorisation as recant.model.ops.gdn_torch (recant/model/ops.py:21-54); see
// gdn_exact.cu for the algebra. Every matmul runs on tcgen05 with M = 128 TMEM lanes by writing the
// products TRANSPOSED, so that the 128-long head dimension is the MMA's M:
//
//   prep  (per chunk x head, parallel)
//     [K; Q] K^T                   M=128 (64 key rows + 64 query rows), N=64, K=dk   -> kk, qk
//     T = (I + strict(beta kk Gamma))^-1      fp32 on CUDA cores (blocked forward substitution)
//     U^T = V^T (T beta)^T          M=dv, N=64, K=64
//     W^T = K^T (T beta e^cum r_k)^T M=dk, N=64, K=64
//   state (per sequence x head, sequential over chunks; S^T [dv][dk] fp32 in registers)
//     V'^T = U^T - S^T W^T          M=dv, N=64,  K=dk
//     O^T  = S^T q~^T + V'^T A_qk^T M=dv, N=64,  K=dk then K=64
//     S^T <- gamma S^T + V'^T k~    M=dv, N=dk,  K=64
//
// Raw bf16 q/k/v feed the MMAs directly; the l2norm scales, decays and beta are folded into fp32
// epilogues or into the small bf16 T-derived operands, so the only added roundings are those of
// T beta, W, U, q~, k~, A_qk, the per-chunk S^T operand and V' (measured ~2.4e-3 relative on o).
#include "gdn_fast.cuh"
#include "tmap.cuh"

namespace rb2 {

size_t carve_fast_saved(Carver& c, FastWs& w, int64_t n_seqs, int Hv, int max_chunks) {
  const size_t nch = size_t(max_chunks) * Hv;
  w.err = c.take<int>(1);  // first: every GDN workspace starts with its status word
  w.ct.tok0 = c.take<int>(max_chunks);
  w.ct.len = c.take<int>(max_chunks);
  w.ct.seq = c.take<int>(max_chunks);
  w.ct.seq_chunk0 = c.take<int>(n_seqs + 1);
  w.ct.order = c.take<int>(n_seqs);
  w.ct.n_chunks = c.take<int>(1);
  w.stats = c.take<float>(nch * 512);
  w.tinv = c.take<__nv_bfloat16>(nch * 4096);
  w.aqk = c.take<__nv_bfloat16>(nch * 4096);
  w.w = c.take<__nv_bfloat16>(nch * 8192);
  w.u = c.take<__nv_bfloat16>(nch * 8192);
  w.qt = c.take<__nv_bfloat16>(nch * 8192);
  w.hs = c.take<__nv_bfloat16>(nch * 16384);
  w.vp = c.take<__nv_bfloat16>(nch * 8192);
  return c.bytes();
}

size_t carve_fast_scratch(Carver& c, FastWs& w, int64_t tokens, int Hv, int max_chunks, bool gqa) {
  const size_t nch = size_t(max_chunks) * Hv;
  w.dh = c.take<__nv_bfloat16>(nch * 16384);
  w.dvp = c.take<__nv_bfloat16>(nch * 8192);
  (void)tokens;
  (void)gqa;  // the GQA group sums of dq / dk stay in the chunk backward's tensor memory
  return c.bytes();
}

namespace {

using namespace fast;

// ------------------------------------------------------------------------------------------------
// Triangular inverse T = (I + L)^-1 of a strictly lower 64x64 L, in place (fp32, stride 65): L on
// entry, T on exit. 256 threads. The 16x16 diagonal blocks by forward substitution on CUDA cores;
// the 16x16 blocks below them inside each 32x32 diagonal block as T_10 = -T_11 (L_10 T_00) on CUDA
// cores; the 32x32 bottom-left block as T_BA = -T_B (L_BA T_A) by two tcgen05 MMAs:
//   X = P D   and   Y = P X'   (M = N = K = 64, bf16 operands, fp32 accumulators in TMEM)
// where P is the working matrix at that point (T_A, T_B on the diagonal, L_BA below), D the same
// with L_BA zeroed (block-diagonal T_A, T_B), and X' = X with its top 32 rows zeroed, so that
// X[B][A] = L_BA T_A and Y[B][A] = T_B X[B][A]. ptile, dtile: 8 KB SW128 tiles (1024-aligned);
// TMEM columns [tcol, tcol + 128) are used; bars: two mbarriers (phase 0) for the two MMAs.
// ------------------------------------------------------------------------------------------------
__device__ void inverse_lower64_tc(float* lt, float* xbuf, unsigned char* ptile, unsigned char* dtile, uint32_t tbase,
                                   uint32_t tcol, uint64_t* bars, int* err) {
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31, q4 = w & 3, hh = w >> 2;
  if (w < 4 && l < 16) {  // warp w: diagonal block w by forward substitution, lane = column
    const int o = 16 * w;
    float col[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float t = (i == l) ? 1.f : 0.f;
#pragma unroll
      for (int m = 0; m < i; ++m) t = fmaf(-lt[(o + i) * 65 + o + m], col[m], t);
      col[i] = t;
    }
    __syncwarp(0x0000ffffu);  // every lane has read the block before any lane overwrites it
#pragma unroll
    for (int i = 0; i < 16; ++i) lt[(o + i) * 65 + o + l] = col[i];
  }
  __syncthreads();
  // blocks (1, 0) and (3, 2): X_b = L_{2b+1,2b} T_{2b,2b}, then T_{2b+1,2b} = -T_{2b+1,2b+1} X_b; a thread
  // owns a 2x2 tile (rows 2 r2, 2 r2 + 1, columns 2 cc, 2 cc + 1) of one block
  const int bq = tid >> 6, r2 = (tid >> 3) & 7, cc = tid & 7;
  const int rb = 16 * (2 * bq + 1), cb = 32 * bq;  // block row / column origin
  if (tid < 128) {
    const float* av = lt + (rb + 2 * r2) * 65 + cb;
    const float* bv = lt + cb * 65 + cb + 2 * cc;
    float x00 = 0.f, x01 = 0.f, x10 = 0.f, x11 = 0.f;
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const float a0 = av[m], a1 = av[65 + m], b0 = bv[m * 65], b1 = bv[m * 65 + 1];
      x00 = fmaf(a0, b0, x00);
      x01 = fmaf(a0, b1, x01);
      x10 = fmaf(a1, b0, x10);
      x11 = fmaf(a1, b1, x11);
    }
    float* xo = xbuf + bq * 256 + 2 * r2 * 16 + 2 * cc;
    *reinterpret_cast<float2*>(xo) = make_float2(x00, x01);
    *reinterpret_cast<float2*>(xo + 16) = make_float2(x10, x11);
  }
  __syncthreads();
  if (tid < 128) {
    const float* av = lt + (rb + 2 * r2) * 65 + rb;
    const float* xb = xbuf + bq * 256 + 2 * cc;
    float t00 = 0.f, t01 = 0.f, t10 = 0.f, t11 = 0.f;
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const float a0 = av[m], a1 = av[65 + m];
      const float2 x = *reinterpret_cast<const float2*>(xb + m * 16);
      t00 = fmaf(a0, x.x, t00);
      t01 = fmaf(a0, x.y, t01);
      t10 = fmaf(a1, x.x, t10);
      t11 = fmaf(a1, x.y, t11);
    }
    float* to = lt + (rb + 2 * r2) * 65 + cb + 2 * cc;
    to[0] = -t00;
    to[1] = -t01;
    to[65] = -t10;
    to[66] = -t11;
  }
  __syncthreads();
  // P (all of the working matrix) and D (its block diagonal) as bf16 images, rows i, columns j
  for (int idx = tid; idx < 512; idx += 256) {  // consecutive lanes take consecutive rows: no bank conflicts
    const int i = idx & 63, c8 = (idx >> 6) * 8;
    const float* t = lt + i * 65 + c8;
    const uint4 v = make_uint4(tc::pack_bf16(t[0], t[1]), tc::pack_bf16(t[2], t[3]), tc::pack_bf16(t[4], t[5]),
                               tc::pack_bf16(t[6], t[7]));
    *reinterpret_cast<uint4*>(ptile + tc::sw128_offset(i, c8, 64)) = v;
    *reinterpret_cast<uint4*>(dtile + tc::sw128_offset(i, c8, 64)) = (i >= 32 && c8 < 32) ? make_uint4(0, 0, 0, 0) : v;
  }
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t pa = tc::smem_u32(ptile), da = tc::smem_u32(dtile);
  const uint32_t idesc = tc::idesc_bf16(64, 64, false, true);  // A = P K-major (rows i), B row-major (MN-major)
  if (tid == 0) {
    const uint64_t d_p = tc::desc_kmajor_sw128(pa), d_d = tc::desc_mnmajor_sw128(da, 8192);
#pragma unroll 1
    for (int k0 = 0; k0 < 64; k0 += 16) tc::mma_bf16(tbase + tcol, d_p + (k0 >> 3), d_d + k0 * 8, idesc, k0 > 0);
    tc::mma_commit(&bars[0]);
  }
  tc::mbar_wait(&bars[0], 0, err, 103);
  tc::fence_after_sync();
  {  // X' into the D tile: rows i = 16 q4 + l (lanes l < 16 of an M = 64 accumulator), zero above row 32
    float x[32];
    tc::tmem_ld32(tbase + (uint32_t(32 * q4) << 16) + tcol + 32 * hh, x);
    if (l < 16) {
      const int i = 16 * q4 + l;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 v = i >= 32 ? make_uint4(tc::pack_bf16(x[8 * j], x[8 * j + 1]), tc::pack_bf16(x[8 * j + 2], x[8 * j + 3]),
                                             tc::pack_bf16(x[8 * j + 4], x[8 * j + 5]),
                                             tc::pack_bf16(x[8 * j + 6], x[8 * j + 7]))
                                : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(dtile + tc::sw128_offset(i, 32 * hh + 8 * j, 64)) = v;
      }
    }
  }
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (tid == 0) {
    const uint64_t d_p = tc::desc_kmajor_sw128(pa), d_d = tc::desc_mnmajor_sw128(da, 8192);
#pragma unroll 1
    for (int k0 = 0; k0 < 64; k0 += 16) tc::mma_bf16(tbase + tcol + 64, d_p + (k0 >> 3), d_d + k0 * 8, idesc, k0 > 0);
    tc::mma_commit(&bars[1]);
  }
  tc::mbar_wait(&bars[1], 0, err, 104);
  tc::fence_after_sync();
  if (q4 >= 2 && hh == 0) {  // T_BA = -Y[B][A]: rows 32..63 (quarters 2, 3), columns 0..31
    float y[32];
    tc::tmem_ld32(tbase + (uint32_t(32 * q4) << 16) + tcol + 64, y);
    if (l < 16) {
      float* to = lt + (16 * q4 + l) * 65;
#pragma unroll
      for (int j = 0; j < 32; ++j) to[j] = -y[j];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
}

// ------------------------------------------------------------------------------------------------
// prep: one CTA (256 threads) per (chunk, value head), three CTAs per SM. Thread (w, l): TMEM lane
// r = 32 (w & 3) + l, column half hh = w >> 2 (columns [32 hh, 32 hh + 32) of the 64-wide
// accumulators). 128 TMEM columns: [K;Q] K^T in [0, 128) is read before the inverse's two products
// and then U^T / W^T reuse them. Shared memory: the [K;Q] tile, whose Q rows (bytes [8K, 16K) and
// [24K, 32K): rows 64-127 of both 64-column slabs) are free once the [K;Q] K^T product is done and
// hold first the inverse's operand tiles and then T beta and T beta e^cum r_k; V; L / T in place
// (fp32). Only the backward walk takes a q~ tile; the forward walk reads the caller's q rows and both
// walks the caller's k rows, with the per-token factors f_q, f_k kept in the stats.
// ------------------------------------------------------------------------------------------------
constexpr int kPrepSmem = 32768 + 16384 + 64 * 65 * 4 + 512 * 4 + 6 * 64 * 4 + 2048;

__global__ void __launch_bounds__(256, 3) fast_prep_kernel(GdnProblem p, FastWs ws, const __grid_constant__ CUtensorMap map_q,
                                                           const __grid_constant__ CUtensorMap map_k,
                                                           const __grid_constant__ CUtensorMap map_v) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = align1024(smem_raw);
  unsigned char* kq = sm;                  // [K;Q] K-major SW128, 128 rows x 128   (32 KB)
  unsigned char* vt = kq + 32768;          // V, 64 rows x 128 (as MN-major A)     (16 KB)
  unsigned char* tb1 = kq + 8192;          // over Q, slab 0: P, then T diag(beta)                  (8 KB)
  unsigned char* tb2 = kq + 24576;         // over Q, slab 1: D / X', then T diag(beta e^cum rk)   (8 KB)
  float* lt = reinterpret_cast<float*>(vt + 16384);  // L, then T (fp32 64 x 65)
  float* xbuf = lt + 64 * 65;
  float* cum = xbuf + 512;
  float* rq = cum + 64;
  float* rk = rq + 64;
  float* beta = rk + 64;
  float* ecum = beta + 64;
  float* gv = ecum + 64;
  __shared__ uint64_t bar[5];  // [K;Q] K^T, U/W, loads, the inverse's two products
  __shared__ uint32_t tmem_base;

  const int ci = blockIdx.x, h = blockIdx.y;
  const int t0 = ws.ct.tok0[ci], L = ws.ct.len[ci];  // len 0: past the last chunk (the grid is max_chunks)
  if (L <= 0) return;
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int r = 32 * (w & 3) + l, hh = w >> 2, c0 = 32 * hh;
  const int hk = h / p.group;
  const int64_t ch = int64_t(ci) * p.Hv + h;

  if (w == 0) {
    tc::tmem_alloc(&tmem_base, 128);
    tc::tmem_relinquish();
  }
  if (tid == 0) {  // k, q, v rows of the chunk by TMA
    for (int b = 0; b < 5; ++b) tc::mbar_init(&bar[b], 1);
    tc::fence_mbar_init();
    tc::mbar_expect_tx(&bar[2], 3 * 16384);
    tc::tma_rows128(kq, 16384, 0, &map_k, hk, t0, &bar[2]);
    tc::tma_rows128(kq, 16384, 64, &map_q, hk, t0, &bar[2]);
    tc::tma_rows128(vt, 8192, 0, &map_v, h, t0, &bar[2]);
  }
  // per-token g and beta: loaded into registers now, stored to shared memory after the TMA wait, so
  // that their latency overlaps the row loads instead of holding up the barrier-init sync
  float g_r = 0.f, beta_r = 0.f;
  if (tid < 64 && tid < L) {
    g_r = p.g[int64_t(t0 + tid) * p.Hv + h];
    beta_r = __bfloat162float(static_cast<const bf16*>(p.beta)[int64_t(t0 + tid) * p.Hv + h]);
  }
  __syncthreads();  // barrier init visible
  tc::mbar_wait(&bar[2], 0, ws.err, 100);
  if (tid < 64) {
    gv[tid] = g_r;
    beta[tid] = beta_r;
  }
  if (L < 64) {  // rows past the end of the sequence
    tc::zero_rows_tail(kq, 16384, 0, L, 256);
    tc::zero_rows_tail(kq, 16384, 64, L, 256);
    tc::zero_rows_tail(vt, 8192, 0, L, 256);
  }
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  const uint32_t lane_addr = tbase + (uint32_t(32 * (w & 3)) << 16) + c0;
  if (tid == 0) {  // [K;Q][K;Q]^T: M=128, N=128, K=128 -> TMEM cols [0, 128)
    const uint64_t d_kq = tc::desc_kmajor_sw128(tc::smem_u32(kq));
    const uint32_t idesc = tc::idesc_bf16(128, 128, false, false);
#pragma unroll
    for (int k0 = 0; k0 < 128; k0 += 16) {
      const uint32_t off = ((k0 >> 6) * 16384 + (k0 & 63) * 2) >> 4;
      tc::mma_bf16(tbase, d_kq + off, d_kq + off, idesc, k0 > 0);
    }
    tc::mma_commit(&bar[0]);
  }
  if (w == 0) {  // cum = cumulative sum of g in double (the reference's fp32 cumsum accumulates in double)
    double lo = gv[l], hi = gv[32 + l];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const double tl = __shfl_up_sync(0xffffffffu, lo, off), th = __shfl_up_sync(0xffffffffu, hi, off);
      if (l >= off) { lo += tl; hi += th; }
    }
    hi += __shfl_sync(0xffffffffu, lo, 31);
    cum[l] = float(lo);
    cum[32 + l] = float(hi);
  }
  tc::mbar_wait(&bar[0], 0, ws.err, 101);
  tc::fence_after_sync();
  // lane r of the accumulator: rows 0-63 = k_i . [k; q], rows 64-127 = q_i . [k; q]; this thread's
  // columns c0..c0+31 of the first 64 (K K^T and Q K^T). The squared norms are diagonals: |k_i|^2 at
  // (i, i), |q_i|^2 at (64 + i, 64 + i), i.e. column 32 q4 + l of lane 32 q4 + l.
  float row[32];
  tc::tmem_ld32(lane_addr, row);
  {
    const int q4 = w & 3;
    float dg[32];
    bool mine = false;
    if (q4 < 2 && hh == q4) {
#pragma unroll
      for (int j = 0; j < 32; ++j) dg[j] = row[j];
      mine = true;
    } else if (q4 >= 2 && hh == 0) {
      tc::tmem_ld32(tbase + (uint32_t(32 * q4) << 16) + 32 * q4, dg);
      mine = true;
    }
    if (mine) {
      float d = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) d = j == l ? dg[j] : d;
      const float rs = rsqrtf(d + 1e-6f);
      if (r < 64) rk[r] = rs; else rq[r - 64] = rs;
    }
  }
  __syncthreads();  // cum, rk, rq
  if (tid < 64) ecum[tid] = __expf(cum[tid]);
  float* st = ws.stats + ch * 512;
  if (tid < 64) {  // stats: cum, r_q, r_k, beta, the per-token factors f_q of q~ and f_k of k~, and the
                   // chunk backward's decay factors e^cum, e^(cum_last - cum) (accurate expf)
    st[tid] = cum[tid]; st[64 + tid] = rq[tid]; st[128 + tid] = rk[tid]; st[192 + tid] = beta[tid];
    st[256 + tid] = p.scale * rq[tid] * __expf(cum[tid]);
    st[320 + tid] = __expf(cum[63] - cum[tid]) * rk[tid];
    st[384 + tid] = expf(cum[tid]);
    st[448 + tid] = expf(cum[63] - cum[tid]);
    // per token j, c_j log2(e) - log2(r_k,j), so that r_k,j e^(c_i - c_j) = 2^(c_i log2(e) - that) in the
    // L / A_qk build below (into g's place: the cumulative sum has consumed it)
    gv[tid] = cum[tid] * kLog2e - __log2f(rk[tid]);
  }
  // q~ rows for the backward walk now (the Q rows' shared memory is reused below): half-warp per row,
  // 8 elements per lane
  for (int row_ = w * 2 + (l >> 4); row_ < 64; row_ += 16) {
    const int c8 = (l & 15) * 8;
    const uint4 x = *reinterpret_cast<const uint4*>(kq + tc::sw128_offset(64 + row_, c8, 128));
    const float f = p.scale * rq[row_] * __expf(cum[row_]);
    const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = tc::pack_bf16(bf_lo(xs[j]) * f, bf_hi(xs[j]) * f);
    *reinterpret_cast<uint4*>(img(ws.qt + ch * 8192) + tc::sw128_offset(row_, c8, 64)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();  // the per-token exponents in gv
  uint32_t apk[16];  // A_qk row i (bf16 pairs), stored after the proxy fence below
  {
    // the masked elements (j > i) may overflow the power of two; they are selected away, not used
    const int i = r & 63;
    const float ci2 = cum[i] * kLog2e;
    float ex[32];
#pragma unroll
    for (int j4 = 0; j4 < 32; j4 += 4) {
      const float4 e4 = *reinterpret_cast<const float4*>(gv + c0 + j4);
      ex[j4] = ex2_approx(ci2 - e4.x);
      ex[j4 + 1] = ex2_approx(ci2 - e4.y);
      ex[j4 + 2] = ex2_approx(ci2 - e4.z);
      ex[j4 + 3] = ex2_approx(ci2 - e4.w);
    }
    if (r < 64) {
      const float bi = beta[i] * rk[i];
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const int j = c0 + jj;
        lt[i * 65 + j] = j < i ? bi * row[jj] * ex[jj] : 0.f;
      }
    } else {
      const float si = p.scale * rq[i];
#pragma unroll
      for (int jj = 0; jj < 32; jj += 2) {
        const int j = c0 + jj;
        const float a = j <= i ? si * row[jj] * ex[jj] : 0.f;
        const float b = j + 1 <= i ? si * row[jj + 1] * ex[jj + 1] : 0.f;
        apk[jj >> 1] = tc::pack_bf16(a, b);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();  // L complete; the Q rows and the [K;Q] K^T accumulator are consumed
  inverse_lower64_tc(lt, xbuf, tb1, tb2, tbase, 0, &bar[3], ws.err);
  {
    const int i = tid & 63, which = (tid >> 6) & 1, m0 = 32 * (tid >> 7);
    unsigned char* dst = which == 0 ? tb1 : tb2;
#pragma unroll
    for (int mb = 0; mb < 32; mb += 8) {
      uint32_t pk[4];
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const int m = m0 + mb + j;
        float f0 = lt[i * 65 + m] * beta[m], f1 = lt[i * 65 + m + 1] * beta[m + 1];
        if (which) { f0 *= ecum[m] * rk[m]; f1 *= ecum[m + 1] * rk[m + 1]; }
        pk[j >> 1] = tc::pack_bf16(f0, f1);
      }
      *reinterpret_cast<uint4*>(dst + tc::sw128_offset(i, m0 + mb, 64)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
  tc::fence_proxy_async();
  __syncthreads();
  tc::fence_after_sync();
  if (tid == 0) {
    // U^T = V^T (T beta)^T: A = V as MN-major (M = dv, K = tok), B = tb1 K-major (N = 64, K = 64)
    // W^T = K^T (T beta e^cum rk)^T: A = rows 0-63 of [K;Q] as MN-major (slab stride 16 KB)
    const uint32_t idesc = tc::idesc_bf16(128, 64, true, false);
    const uint64_t d_v = tc::desc_mnmajor_sw128(tc::smem_u32(vt), 8192), d_k = tc::desc_mnmajor_sw128(tc::smem_u32(kq), 16384),
                   d_1 = tc::desc_kmajor_sw128(tc::smem_u32(tb1)), d_2 = tc::desc_kmajor_sw128(tc::smem_u32(tb2));
#pragma unroll
    for (int k0 = 0; k0 < 64; k0 += 16) {
      tc::mma_bf16(tbase + 0, d_v + k0 * 8, d_1 + (k0 >> 3), idesc, k0 > 0);
      tc::mma_bf16(tbase + 64, d_k + k0 * 8, d_2 + (k0 >> 3), idesc, k0 > 0);
    }
    tc::mma_commit(&bar[1]);
  }
  // workspace images of A_qk and T (global stores kept behind the proxy fence above)
  if (r >= 64) {
    unsigned char* dst = img(ws.aqk + ch * 4096);
    const int i = r & 63;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(dst + tc::sw128_offset(i, c0 + 8 * j, 64)) =
          make_uint4(apk[4 * j], apk[4 * j + 1], apk[4 * j + 2], apk[4 * j + 3]);
  }
  for (int idx = tid; idx < 512; idx += 256) {  // consecutive lanes take consecutive rows: no bank conflicts
    const int i = idx & 63, c8 = (idx >> 6) * 8;
    const float* t = lt + i * 65 + c8;
    *reinterpret_cast<uint4*>(img(ws.tinv + ch * 4096) + tc::sw128_offset(i, c8, 64)) =
        make_uint4(tc::pack_bf16(t[0], t[1]), tc::pack_bf16(t[2], t[3]), tc::pack_bf16(t[4], t[5]),
                   tc::pack_bf16(t[6], t[7]));
  }
  tc::mbar_wait(&bar[1], 0, ws.err, 102);
  tc::fence_after_sync();
  {
    // lane r = dv (for U) or dk (for W); tokens c0..c0+31
    float tmp[32];
    tc::tmem_ld32(lane_addr + 0, tmp);
    store_cols32(ws.u + ch * 8192, 128, r, c0, 64, tmp);
    tc::tmem_ld32(lane_addr + 64, tmp);
    store_cols32_img(img(ws.w + ch * 8192), 64, r, c0, tmp);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (w == 0) tc::tmem_dealloc(tbase, 128);
}

// ------------------------------------------------------------------------------------------------
// forward state walk: one CTA (256 threads) per (sequence, value head)
//   thread (w, l): TMEM lane / dv row r = 32 (w & 3) + l, dk half hh = w >> 2
// ------------------------------------------------------------------------------------------------
constexpr int kStageBytes = 16384 * 4 + 8192 + 2048;  // W, q, k, U, A_qk, stats (1024-byte multiple)
constexpr int kStateSmem = 32768 + 16384 + 16384 + 2 * kStageBytes + 2048;

// The caller's q and k rows come by TMA and are used raw: q~ = f_q q and k~ = f_k k with per-token
// f_q = scale r_q e^cum and f_k = r_k e^(cum_last - cum) (the prep's l2-norm and decay factors), so
// S^T q~^T = (S^T q^T) diag(f_q) is scaled in the output epilogue and V'^T k~ = (V'^T diag(f_k)) k
// takes a second, scaled V'^T tile.
struct FwdStage {
  unsigned char* wt;   // [W; q]: one 128-row K-major tile (slab stride 16 KB), rows 0-63 W, 64-127 the
                       // caller's q rows, so S^T [W; q]^T is one N = 128 product              32 KB
  unsigned char* kt;   // k   64 x 128 (used MN-major: N = dk) 16 KB
  bf16* us;            // U plain [64][128]                    16 KB
  unsigned char* at;   // A_qk 64 (i) x 64 (j)                  8 KB
  float* cum;          // stats: cum, r_q, r_k, beta, f_q, f_k (64 floats each)
};

__device__ __forceinline__ FwdStage fwd_stage(unsigned char* base, int stg) {
  unsigned char* b = base + stg * kStageBytes;
  FwdStage st;
  st.wt = b;
  st.kt = b + 32768;
  st.us = reinterpret_cast<bf16*>(b + 49152);
  st.at = b + 65536;
  st.cum = reinterpret_cast<float*>(b + 65536 + 8192);
  return st;
}

// One thread: the chunk's q, k rows by TMA and its workspace tile images (W, U, A_qk) and stats by
// bulk copies into a stage, counted on `bar`.
__device__ __forceinline__ void fwd_issue(const FwdStage& st, const FastWs& ws, int64_t ch, int walk, int hk, int t0,
                                          const CUtensorMap* map_q, const CUtensorMap* map_k, uint64_t* bar) {
  const uint32_t bytes = 16384 * 2 + 1536 + (walk == 0 ? 16384 + 8192 : 0) + (walk != 2 ? 16384 : 0);
  tc::fence_proxy_async();  // the stage's previous generic reads are ordered before these writes
  tc::mbar_expect_tx(bar, bytes);
  tc::bulk_load(st.wt, ws.w + ch * 8192, 8192, bar);                  // W image slab 0 -> rows 0-63
  tc::bulk_load(st.wt + 16384, ws.w + ch * 8192 + 4096, 8192, bar);   // slab 1
  tc::tma_rows128(st.kt, 8192, 0, map_k, hk, t0, bar);
  if (walk == 0) {  // outputs need q and A_qk
    tc::tma_rows128(st.wt, 16384, 64, map_q, hk, t0, bar);
    tc::bulk_load(st.at, ws.aqk + ch * 4096, 8192, bar);
  }
  if (walk != 2) tc::bulk_load(st.us, ws.u + ch * 8192, 16384, bar);
  tc::bulk_load(st.cum, ws.stats + ch * 512, 1536, bar);
}

__global__ void __launch_bounds__(256, 1) fast_state_fwd_kernel(GdnProblem p, FastWs ws, bf16* __restrict__ o,
                                                                 float* __restrict__ hT,
                                                                 const __grid_constant__ CUtensorMap map_q,
                                                                 const __grid_constant__ CUtensorMap map_k) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = align1024(smem_raw);
  unsigned char* st = sm;                   // S^T bf16, K-major 128 rows (dv) x 128 (dk)   32 KB
  unsigned char* vpt = st + 32768;          // V'^T 128 rows (dv) x 64 (tok)                16 KB
  unsigned char* vpk = vpt + 16384;         // V'^T diag(f_k), the S update's operand      16 KB
  unsigned char* stages = vpk + 16384;      // 2 x FwdStage
  __shared__ uint64_t bar[2];
  __shared__ uint64_t ldbar[2];   // stage loads
  __shared__ uint32_t tmem_base;

  const int h = blockIdx.x, s = ws.ct.order[blockIdx.y], hk = h / p.group;  // longest sequences first
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int r = 32 * (w & 3) + l, hh = w >> 2;
  if (w == 0) tc::tmem_alloc(&tmem_base, 512);
  const int c0 = ws.ct.seq_chunk0[s], c1 = ws.ct.seq_chunk0[s + 1];
  if (tid == 0) {
    tc::mbar_init(&bar[0], 1);
    tc::mbar_init(&bar[1], 1);
    tc::mbar_init(&ldbar[0], 1);
    tc::mbar_init(&ldbar[1], 1);
    tc::fence_mbar_init();
    if (c0 < c1)
      fwd_issue(fwd_stage(stages, 0), ws, int64_t(c0) * p.Hv + h, p.walk, hk, ws.ct.tok0[c0], &map_q, &map_k, &ldbar[0]);
  }
  // S^T[r][dk] for dk in [64 hh, 64 hh + 64): S[dk][r] of the [dk][dv] state
  float S[64];
  const int64_t sbase = (int64_t(s) * p.Hv + h) * 16384;
#pragma unroll
  for (int j = 0; j < 64; ++j)
    S[j] = p.walk == 2 ? (64 * hh + j == r ? 1.f : 0.f) : (p.h0 ? p.h0[sbase + (64 * hh + j) * 128 + r] : 0.f);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  const uint32_t lane_addr = tbase + (uint32_t(32 * (w & 3)) << 16);
  const bool outs = p.walk == 0;  // per-chunk outputs (o, S, V') only in the normal walk
  uint32_t phase = 0;
  for (int ci = c0; ci < c1; ++ci) {
    const int64_t ch = int64_t(ci) * p.Hv + h;
    const int t0 = ws.ct.tok0[ci], L = ws.ct.len[ci];
    const int stg = (ci - c0) & 1;
    const FwdStage cur = fwd_stage(stages, stg);
    if (tid == 0 && ci + 1 < c1)
      fwd_issue(fwd_stage(stages, stg ^ 1), ws, ch + p.Hv, p.walk, hk, ws.ct.tok0[ci + 1], &map_q, &map_k,
                &ldbar[stg ^ 1]);
    tc::mbar_wait(&ldbar[stg], ((ci - c0) >> 1) & 1, ws.err, 110);
    if (L < 64) {  // the caller's rows past the end of the sequence (another sequence's, or the TMA fill)
      tc::zero_rows_tail(cur.kt, 8192, 0, L, 256);
      if (outs) tc::zero_rows_tail(cur.wt, 16384, 64, L, 256);
    }
    // S^T (bf16) -> smem operand and -> workspace (state entering this chunk)
    {
      uint32_t pk[32];
#pragma unroll
      for (int j = 0; j < 64; j += 2) pk[j >> 1] = tc::pack_bf16(S[j], S[j + 1]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 v4 = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        *reinterpret_cast<uint4*>(st + tc::sw128_offset(r, 64 * hh + 8 * j, 128)) = v4;
      }
    }
    tc::fence_proxy_async();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0) {
      // [D_vp D_o] = S^T [W; q]^T: D_vp in columns [0,64), D_o = S^T q^T (scaled by f_q later) in [64,128);
      // M=128, N=128 (N=64, W only, without outputs), K=128
      const uint32_t idesc = tc::idesc_bf16(128, outs ? 128 : 64, false, false);
      const uint64_t d_s = tc::desc_kmajor_sw128(tc::smem_u32(st)), d_wq = tc::desc_kmajor_sw128(tc::smem_u32(cur.wt));
#pragma unroll
      for (int k0 = 0; k0 < 128; k0 += 16) {
        const uint32_t off = ((k0 >> 6) * 16384 + (k0 & 63) * 2) >> 4;  // both operands: 16 KB slabs
        tc::mma_bf16(tbase + 0, d_s + off, d_wq + off, idesc, k0 > 0);
      }
      tc::mma_commit(&bar[0]);
      if (outs) {  // the state entering the chunk: the S^T tile is its workspace image
        tc::bulk_store(ws.hs + ch * 16384, st, 32768);
        tc::bulk_commit();
      }
    }
    tc::mbar_wait(&bar[0], phase, ws.err, 111);
    tc::fence_after_sync();
    {
      // V'^T[r][tok] = U[tok][r] - D_vp[r][tok] for tok in [32 hh, 32 hh + 32)
      float x[32];
      tc::tmem_ld32(lane_addr + 32 * hh, x);
      uint32_t pk[16];
      if (p.walk == 2) {  // transition: U = 0
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = -x[j];
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = __bfloat162float(cur.us[(32 * hh + j) * 128 + r]) - x[j];
      }
#pragma unroll
      for (int j = 0; j < 32; j += 2) pk[j >> 1] = tc::pack_bf16(x[j], x[j + 1]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(vpt + tc::sw128_offset(r, 32 * hh + 8 * j, 128)) =
            make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
#pragma unroll
      float fk[32];
      lds_vec(cur.cum + 320 + 32 * hh, fk);  // f_k = r_k e^(cum_last - cum)
#pragma unroll
      for (int j = 0; j < 32; j += 2) pk[j >> 1] = tc::pack_bf16(x[j] * fk[j], x[j + 1] * fk[j + 1]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(vpk + tc::sw128_offset(r, 32 * hh + 8 * j, 128)) =
            make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (tid == 0) {
      // D_o2 = V'^T A_qk^T (cols [128, 192); M=128, N=64, K=64); D_s = (V'^T diag(f_k)) k (M=128, N=128, K=64,
      // k MN-major)
      const uint64_t d_v = tc::desc_kmajor_sw128(tc::smem_u32(vpt)), d_vk = tc::desc_kmajor_sw128(tc::smem_u32(vpk)),
                     d_a = tc::desc_kmajor_sw128(tc::smem_u32(cur.at)), d_k = tc::desc_mnmajor_sw128(tc::smem_u32(cur.kt), 8192);
      const uint32_t id_o = tc::idesc_bf16(128, 64, false, false);
      const uint32_t id_s = tc::idesc_bf16(128, 128, false, true);
#pragma unroll
      for (int k0 = 0; k0 < 64; k0 += 16) {
        if (outs) tc::mma_bf16(tbase + 128, d_v + (k0 >> 3), d_a + (k0 >> 3), id_o, k0 > 0);
        tc::mma_bf16(tbase + 256, d_vk + (k0 >> 3), d_k + k0 * 8, id_s, k0 > 0);
      }
      tc::mma_commit(&bar[1]);
      if (outs) {  // V'^T [dv][tok]: the tile is the workspace image
        tc::bulk_store(ws.vp + ch * 8192, vpt, 16384);
        tc::bulk_commit();
      }
    }
    tc::mbar_wait(&bar[1], phase, ws.err, 112);
    tc::fence_after_sync();
    float ox[32];  // o rows of this chunk, stored after the barrier below (stores ahead of a fence stall it)
    {
      float x[32];
      if (outs) {  // o^T = (S^T q^T) diag(f_q) + V'^T A_qk^T
        tc::tmem_ld32(lane_addr + 64 + 32 * hh, ox);
        tc::tmem_ld32(lane_addr + 128 + 32 * hh, x);
        float fq[32];
        lds_vec(cur.cum + 256 + 32 * hh, fq);  // f_q
#pragma unroll
        for (int j = 0; j < 32; ++j) ox[j] = fmaf(fq[j], ox[j], x[j]);
      }
      const float gamma = expf(cur.cum[63]);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tc::tmem_ld32(lane_addr + 256 + 64 * hh + 32 * half, x);
#pragma unroll
        for (int j = 0; j < 32; ++j) S[32 * half + j] = fmaf(gamma, S[32 * half + j], x[j]);
      }
    }
    if (tid == 0) tc::bulk_wait_read();  // the S^T and V'^T tiles are rewritten next step
    tc::fence_before_sync();
    __syncthreads();
    if (outs) store_cols32(o + (int64_t(t0) * p.Hv + h) * 128, p.Hv * 128, r, 32 * hh, L, ox);
    phase ^= 1;
  }
  if (hT) {
#pragma unroll
    for (int j = 0; j < 64; ++j) hT[sbase + (64 * hh + j) * 128 + r] = S[j];
  }
  if (tid == 0) tc::bulk_wait_all();
  tc::fence_before_sync();
  __syncthreads();
  if (w == 0) tc::tmem_dealloc(tbase, 512);
}

template <typename K>
int smem_attr(K kernel, int bytes) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return RB2_ECUDA;
  }
  return RB2_OK;
}

}  // namespace

void fast_workspace_split(int64_t tokens, int64_t n_seqs, int Hk, int Hv, int max_chunks, size_t* saved,
                          size_t* scratch) {
  FastWs w;
  Carver a(nullptr), b(nullptr);
  *saved = carve_fast_saved(a, w, n_seqs, Hv, max_chunks);
  *scratch = carve_fast_scratch(b, w, tokens, Hv, max_chunks, Hk != Hv);
}

static int check_err_word(const FastWs& w, cudaStream_t s, bool sync) {
  (void)w; (void)s; (void)sync;
  return RB2_OK;
}

int fast_forward(const GdnProblem& p, void* wsp, void* o, float* hT, cudaStream_t s) {
  Carver c(wsp);
  FastWs w;
  carve_fast_saved(c, w, p.n_seqs, p.Hv, p.max_chunks);
  int rc = RB2_OK;
  if (p.stages & 1) {
    if ((rc = launch_chunk_table(p, w.ct, s))) return rc;
    RB2_CUDA(cudaMemsetAsync(w.err, 0, sizeof(int), s), "gdn fast: clear status");
  }
  if ((p.stages & 1) && p.max_chunks > 0) {
    if ((rc = smem_attr(fast_prep_kernel, kPrepSmem))) return rc;
    // all of the SM's unified memory as shared memory, so that three prep CTAs fit on one SM
    RB2_CUDA(cudaFuncSetAttribute(fast_prep_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100),
             "gdn fast prep: carveout");
    ProfScope ps_("gdn_fast_prep", s);
    CUtensorMap mq, mk, mv;
    if ((rc = make_rows_map(&mq, p.q, p.tokens, p.Hk)) || (rc = make_rows_map(&mk, p.k, p.tokens, p.Hk)) ||
        (rc = make_rows_map(&mv, p.v, p.tokens, p.Hv)))
      return rc;
    fast_prep_kernel<<<dim3(p.max_chunks, p.Hv), 256, kPrepSmem, s>>>(p, w, mq, mk, mv);
    RB2_CHECK_LAUNCH("gdn fast prep");
  }
  if (!(p.stages & 2)) return RB2_OK;
  if ((rc = smem_attr(fast_state_fwd_kernel, kStateSmem))) return rc;
  {
    ProfScope ps_("gdn_fast_state_fwd", s);
    CUtensorMap mq, mk;
    if ((rc = make_rows_map(&mq, p.q, p.tokens, p.Hk)) || (rc = make_rows_map(&mk, p.k, p.tokens, p.Hk))) return rc;
    fast_state_fwd_kernel<<<dim3(p.Hv, unsigned(p.n_seqs)), 256, kStateSmem, s>>>(p, w, static_cast<bf16*>(o), hT, mq,
                                                                                    mk);
    RB2_CHECK_LAUNCH("gdn fast state fwd");
  }
  return check_err_word(w, s, false);
}


}  // namespace rb2
