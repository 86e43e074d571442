// Chunked Gated DeltaNet backward on tcgen05 (the autograd of recant.model.ops.gdn_torch,
// recant/model/ops.py:21-54, written out by hand).
//
// Per chunk, with S the state entering it and dS the gradient of the state leaving it:
//   reversed walk (per sequence x head, sequential):
//     dV'^T = dO^T A_qk + dS^T k~^T                         M=dv, N=64, K=64 and K=dk
//     dS^T  <- gamma dS^T + dO^T q~ - dV'^T W               M=dv, N=dk, K=64 (negated A)
//   chunk backward (per chunk x head, parallel), transposed so d is the MMA's M wherever the
//   output is [d][tok]; 64x64 token-by-token products use M=64 (rows in lanes 0-15 of each
//   32-lane quarter):
//     dq~^T = S dO^T, dW^T = -S dV'^T, dk~^T = dS V'^T, dA_qk = dO V'^T      (G1)
//     dT = dV' (beta V)^T + dW (beta e^cum r_k K)^T, dBv^T = dV'^T T, dBk^T = dW^T T   (G2)
//     Y = T^T dT (G3);  dL = -Y T^T (G4)
//     dk^ += diag(beta) P k^ + P^T diag(beta) k^ + Qm^T q^,  dq^ += Qm k^   (G5)
//       with P = dL * Gamma (strictly lower) and Qm = dA_qk * Gamma
//   then the decay factors, beta, the cumulative gate (reverse cumsum -> dg) and the l2norm.
#include "gdn_fast.cuh"
#include "tmap.cuh"

namespace rb2 {
namespace {

using namespace fast;

__device__ __forceinline__ float tile_elem(const unsigned char* tile, int rows, int r, int k) {
  return __bfloat162float(*reinterpret_cast<const bf16*>(tile + tc::sw128_offset(r, k, rows)));
}

__device__ __forceinline__ void sync_for_mma() {
  tc::fence_proxy_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
}

// ------------------------------------------------------------------------------------------------
// reversed state walk: one CTA (256 threads) per (sequence, value head); thread = (dv row, dk half)
// ------------------------------------------------------------------------------------------------
constexpr int kBStageBytes = 16384 * 4 + 8192 + 2048;  // dO, k, q~, W, A_qk, stats (1024-byte multiple)
constexpr int kBStateSmem = 32768 + 16384 + 2 * kBStageBytes + 2048;

// The caller's k rows are used raw, as in the forward walk: dS^T k~^T = (dS^T k^T) diag(f_k) is scaled
// in the dV' epilogue with the prep's f_k; q~ comes from the prep as a tile image (scaling dO instead
// would put a pass over it on the walk's critical path).
struct BwdStage {
  unsigned char* dot;  // dO rows tok (64) x dv
  unsigned char* kt;   // k rows tok x dk (the caller's)
  unsigned char* qt;   // q~ rows (tile image)
  unsigned char* wt;   // W
  unsigned char* at;   // A_qk rows i x c
  float* cum;          // stats: cum, r_q, r_k, beta, f_q, f_k
};

__device__ __forceinline__ BwdStage bwd_stage(unsigned char* base, int stg) {
  unsigned char* b = base + stg * kBStageBytes;
  BwdStage st;
  st.dot = b;
  st.kt = b + 16384;
  st.qt = b + 32768;
  st.wt = b + 49152;
  st.at = b + 65536;
  st.cum = reinterpret_cast<float*>(b + 65536 + 8192);
  return st;
}

// Thread 0: the chunk's dO and k rows by TMA (rows past the sequence are zeroed after the wait)
// and the workspace tile images (q~, W, A_qk) and stats by bulk copies, counted on `bar`.
__device__ __forceinline__ void bwd_issue(const BwdStage& st, const GdnProblem& p, const FastWs& ws,
                                          const CUtensorMap* map_do, const CUtensorMap* map_k, int ci, int h,
                                          uint64_t* bar) {
  const int64_t ch = int64_t(ci) * p.Hv + h;
  const int t0 = ws.ct.tok0[ci], hk = h / p.group;
  if (threadIdx.x == 0) {
    tc::fence_proxy_async();
    tc::mbar_expect_tx(bar, 4 * 16384 + 8192 + 1536);
    tc::tma_rows128(st.dot, 8192, 0, map_do, h, t0, bar);
    tc::tma_rows128(st.kt, 8192, 0, map_k, hk, t0, bar);
    tc::bulk_load(st.qt, ws.qt + ch * 8192, 16384, bar);
    tc::bulk_load(st.wt, ws.w + ch * 8192, 16384, bar);
    tc::bulk_load(st.at, ws.aqk + ch * 4096, 8192, bar);
    tc::bulk_load(st.cum, ws.stats + ch * 512, 1536, bar);
  }
}

__global__ void __launch_bounds__(256, 1) fast_state_bwd_kernel(GdnProblem p, FastWs ws, const __grid_constant__ CUtensorMap map_do,
                                                                 const float* __restrict__ dhT, float* __restrict__ dh0,
                                                                 const __grid_constant__ CUtensorMap map_k) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = align1024(smem_raw);
  unsigned char* dst = sm;              // dS^T bf16, rows dv (128) x dk               32 KB
  unsigned char* dvt = dst + 32768;     // dV'^T rows dv x tok                          16 KB
  unsigned char* stages = dvt + 16384;  // 2 x BwdStage
  __shared__ uint64_t bar[2];
  __shared__ uint64_t ldbar[2];   // stage loads (bulk part)
  __shared__ uint32_t tmem_base;

  const int h = blockIdx.x, s = ws.ct.order[blockIdx.y];  // longest sequences first
  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int r = 32 * (w & 3) + l, hh = w >> 2;
  if (w == 0) tc::tmem_alloc(&tmem_base, 512);
  if (tid == 0) {
    tc::mbar_init(&bar[0], 1);
    tc::mbar_init(&bar[1], 1);
    tc::mbar_init(&ldbar[0], 1);
    tc::mbar_init(&ldbar[1], 1);
    tc::fence_mbar_init();
  }
  const int c0 = ws.ct.seq_chunk0[s], c1 = ws.ct.seq_chunk0[s + 1];
  if (c0 < c1) bwd_issue(bwd_stage(stages, 0), p, ws, &map_do, &map_k, c1 - 1, h, &ldbar[0]);
  float dS[64];
  const int64_t sbase = (int64_t(s) * p.Hv + h) * 16384;
#pragma unroll
  for (int j = 0; j < 64; ++j) dS[j] = dhT ? dhT[sbase + (64 * hh + j) * 128 + r] : 0.f;
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  const uint32_t lane_addr = tbase + (uint32_t(32 * (w & 3)) << 16);
  uint32_t phase = 0;
  for (int ci = c1 - 1; ci >= c0; --ci) {
    const int64_t ch = int64_t(ci) * p.Hv + h;
    const int stg = (c1 - 1 - ci) & 1;
    const BwdStage cur = bwd_stage(stages, stg);
    if (ci - 1 >= c0) bwd_issue(bwd_stage(stages, stg ^ 1), p, ws, &map_do, &map_k, ci - 1, h, &ldbar[stg ^ 1]);
    tc::mbar_wait(&ldbar[stg], ((c1 - 1 - ci) >> 1) & 1, ws.err, 120);
    const int Lc = ws.ct.len[ci];
    if (Lc < 64) {  // dO and k rows past the sequence
      tc::zero_rows_tail(cur.dot, 8192, 0, Lc, 256);
      tc::zero_rows_tail(cur.kt, 8192, 0, Lc, 256);
    }
    {
      uint32_t pk[32];
#pragma unroll
      for (int j = 0; j < 64; j += 2) pk[j >> 1] = tc::pack_bf16(dS[j], dS[j + 1]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 v4 = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
        *reinterpret_cast<uint4*>(dst + tc::sw128_offset(r, 64 * hh + 8 * j, 128)) = v4;
      }
    }
    sync_for_mma();
    if (tid == 0) {
      const uint64_t d_do = tc::desc_mnmajor_sw128(tc::smem_u32(cur.dot), 8192),
                     d_a = tc::desc_mnmajor_sw128(tc::smem_u32(cur.at), 8192), d_ds = tc::desc_kmajor_sw128(tc::smem_u32(dst)),
                     d_k = tc::desc_kmajor_sw128(tc::smem_u32(cur.kt)),
                     d_q = tc::desc_mnmajor_sw128(tc::smem_u32(cur.qt), 8192);
      // dV'^T = dO^T A_qk (A = dO MN-major: M = dv, K = tok; B = A_qk MN-major: N = c, K = i)
      const uint32_t id_a = tc::idesc_bf16(128, 64, true, true);
#pragma unroll
      for (int k0 = 0; k0 < 64; k0 += 16) tc::mma_bf16(tbase + 0, d_do + k0 * 8, d_a + k0 * 8, id_a, k0 > 0);
      // D_k = dS^T k^T into columns [64, 128), scaled by f_k in the epilogue (A = dS^T K-major: M = dv,
      // K = dk; B = k K-major: N = tok, K = dk)
      const uint32_t id_b = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
      for (int k0 = 0; k0 < 128; k0 += 16)
        tc::mma_bf16(tbase + 64, d_ds + (((k0 >> 6) * 16384 + (k0 & 63) * 2) >> 4),
                       d_k + (((k0 >> 6) * 8192 + (k0 & 63) * 2) >> 4), id_b, k0 > 0);
      // D_s = dO^T q~ (A = dO MN-major; B = q~ MN-major: N = dk, K = tok)
      const uint32_t id_s = tc::idesc_bf16(128, 128, true, true);
#pragma unroll
      for (int k0 = 0; k0 < 64; k0 += 16) tc::mma_bf16(tbase + 256, d_do + k0 * 8, d_q + k0 * 8, id_s, k0 > 0);
      tc::mma_commit(&bar[0]);
      if (p.walk == 0) {  // the gradient of the state leaving the chunk: the dS^T tile is its image
        tc::bulk_store(ws.dh + ch * 16384, dst, 32768);
        tc::bulk_commit();
      }
    }
    tc::mbar_wait(&bar[0], phase, ws.err, 121);
    tc::fence_after_sync();
    {
      float x[32], xk[32];  // dV'^T = dO^T A_qk + (dS^T k^T) diag(f_k)
      tc::tmem_ld32(lane_addr + 32 * hh, x);
      tc::tmem_ld32(lane_addr + 64 + 32 * hh, xk);
      float fk[32];
      lds_vec(cur.cum + 320 + 32 * hh, fk);  // f_k
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] = fmaf(fk[j], xk[j], x[j]);
      uint32_t pk[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) pk[j >> 1] = tc::pack_bf16(x[j], x[j + 1]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(dvt + tc::sw128_offset(r, 32 * hh + 8 * j, 128)) =
            make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
    }
    sync_for_mma();
    if (tid == 0) {
      // D_s -= dV'^T W (A = dV'^T K-major: M = dv, K = tok, negated; B = W MN-major: N = dk, K = tok)
      const uint64_t d_v = tc::desc_kmajor_sw128(tc::smem_u32(dvt)), d_w = tc::desc_mnmajor_sw128(tc::smem_u32(cur.wt), 8192);
      const uint32_t id_w = tc::idesc_bf16(128, 128, false, true, true);
#pragma unroll
      for (int k0 = 0; k0 < 64; k0 += 16) tc::mma_bf16(tbase + 256, d_v + (k0 >> 3), d_w + k0 * 8, id_w, true);
      tc::mma_commit(&bar[1]);
      if (p.walk == 0) {  // dV'^T [dv][tok]: the tile is the workspace image
        tc::bulk_store(ws.dvp + ch * 8192, dvt, 16384);
        tc::bulk_commit();
      }
    }
    tc::mbar_wait(&bar[1], phase, ws.err, 122);
    tc::fence_after_sync();
    {
      const float gamma = expf(cur.cum[63]);
      float x[32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tc::tmem_ld32(lane_addr + 256 + 64 * hh + 32 * half, x);
#pragma unroll
        for (int j = 0; j < 32; ++j) dS[32 * half + j] = fmaf(gamma, dS[32 * half + j], x[j]);
      }
    }
    if (tid == 0) tc::bulk_wait_read();  // the dS^T tile is rewritten next step
    tc::fence_before_sync();
    __syncthreads();
    phase ^= 1;
  }
  if (dh0) {
#pragma unroll
    for (int j = 0; j < 64; ++j) dh0[sbase + (64 * hh + j) * 128 + r] = dS[j];
  }
  if (tid == 0) tc::bulk_wait_all();
  tc::fence_before_sync();
  __syncthreads();
  if (w == 0) tc::tmem_dealloc(tbase, 512);
}

// ------------------------------------------------------------------------------------------------
// chunk backward: persistent, one CTA of 512 threads (16 warps) per SM. Thread (w, l): TMEM lane
// quarter q = w & 3, lane r = 32 q + l (head-dim row of an M=128 accumulator; for M=64 accumulators
// lanes l < 16 hold token rows 16 q + l), column quarter cq = w >> 2 (columns [16 cq, 16 cq + 16)).
// Sixteen warps (four per scheduler) hide the latency of the epilogues' shared-memory and TMEM
// traffic; each thread holds 16 columns of an accumulator row, so 128 registers suffice.
// TMEM columns (64-column blocks): G1 writes [K;Q]K^T 0, dq~^T 64, dW^T 128, dk~^T 192, dA_qk 256;
// E1 frees 0, 128, 256; G2 writes dV' V^T 320, dW K^T 0 (the two parts of dT, combined with the
// per-token factors in E2), dBv^T 128, dBk^T 256; G3 Y 0; G4 dL' 128; G5 320 and 0.
// Columns [384, 512) are never written by an MMA: they carry the GQA group's running dq / dk sums
// (fp32) from one value head of the group to the next.
// ------------------------------------------------------------------------------------------------
namespace lay {  // shared-memory map (bytes from the 1024-aligned base)
constexpr int KQ = 0, VT = 32768, DVP = 49152;
constexpr int ST = 65536, DHT = 98304, DOT = 131072, VPT = 147456;           // phase 1
constexpr int DWT = 65536, TT = 114688, DTT = 122880,                        // phase 2 (over phase 1)
              YT = 131072, PB1 = 139264, PB2 = 147456, QB1 = 155648;
constexpr int QB2 = VT;                                                        // over V once consumed
constexpr int DVS = DWT;     // dv rows, bf16 [64][128], from E2 until after G5 is issued
constexpr int KKF = 163840, QKF = KKF + 16640, DAQF = QKF + 16640;             // fp32 [64][65]
constexpr int VEC = DAQF + 16640;                                              // 18 x 64 floats
constexpr int RED = VEC + 18 * 256;                                            // 16 + 5 x 4 x 64 floats
constexpr int STATS = RED + 5 * 1024 + 64;  // the next item's per-token stats, fp32 [8][64], by bulk copy
constexpr int END = STATS + 2048;
}  // namespace lay
constexpr int kBChunkSmem = lay::END + 1024;
constexpr int kBThreads = 512;

// Sum v[0..31] over the 32 lanes; afterwards lane l holds the total of column l.
__device__ __forceinline__ float warp_colsum32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    const int s = 16 >> step, c = 32 >> step;
    const bool up = (lane & s) != 0;
#pragma unroll
    for (int j = 0; j < c / 2; ++j) {
      const float send = up ? v[j] : v[j + c / 2];
      const float keep = up ? v[j + c / 2] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

// Sum v[0..15] over the 32 lanes; afterwards lanes 2c and 2c + 1 hold the total of column c.
__device__ __forceinline__ float warp_colsum16(float (&v)[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int s = 16 >> step, c = 16 >> step;
    const bool up = (lane & s) != 0;
#pragma unroll
    for (int j = 0; j < c / 2; ++j) {
      const float send = up ? v[j] : v[j + c / 2];
      const float keep = up ? v[j + c / 2] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

__device__ __forceinline__ void tmem_ld16f(uint32_t addr, float (&v)[16]) { tc::tmem_ld16(addr, v); }


__global__ void __launch_bounds__(kBThreads, 1) fast_chunk_bwd_kernel(GdnProblem p, FastWs ws, const bf16* __restrict__ d_o,
                                                                 bf16* __restrict__ dq, bf16* __restrict__ dk,
                                                                 bf16* __restrict__ dv, float* __restrict__ dg,
                                                                 bf16* __restrict__ dbeta,
                                                                 const __grid_constant__ CUtensorMap map_q,
                                                                 const __grid_constant__ CUtensorMap map_k,
                                                                 const __grid_constant__ CUtensorMap map_v,
                                                                 const __grid_constant__ CUtensorMap map_do) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = align1024(smem_raw);
  float* kkf = reinterpret_cast<float*>(sm + lay::KKF);
  float* qkf = reinterpret_cast<float*>(sm + lay::QKF);
  float* daqf = reinterpret_cast<float*>(sm + lay::DAQF);
  float* vec = reinterpret_cast<float*>(sm + lay::VEC);
  float *cum = vec, *rq = vec + 64, *rk = vec + 128, *beta = vec + 192, *ecum = vec + 256, *edec = vec + 320,
        *dbeta_acc = vec + 384, *dcum_acc = vec + 448, *dbp = vec + 512 /* [8][64] */, *scal = vec + 1024;
  float* red = reinterpret_cast<float*>(sm + lay::RED);  // [5][4][64]; the first 16 also per-warp partials
  __shared__ uint64_t bar[5];
  __shared__ uint64_t ldbar[3];   // loads: phase-1 tiles and stats (bulk + TMA), T, [K;Q] (TMA)
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  const int q4 = w & 3, cq = w >> 2, r = 32 * q4 + l, c0 = 16 * cq;
  const bool mrow = l < 16;            // this lane holds a row of an M=64 accumulator
  const int i64 = 16 * q4 + l;          // ... and it is token row i64
  // Work: (chunk, key head) groups G = chunk * Hk + key head, each the p.group value heads that share
  // the key head, walked group after group by one CTA (grid-strided over groups) so that the group's
  // dq / dk can be summed in tensor memory. An item is one (chunk, value head); the sequence is
  // advanced incrementally in 32-bit arithmetic (one division per group), and an item's chunk-table
  // entries are read when it becomes the next item, a whole item ahead of their use.
  const int n_groups = *ws.ct.n_chunks * p.Hk;
  struct Item {
    int G, gi, ci, hk, h;  // group, index in the group, chunk, key head, value head
    int t0, L;             // the chunk's first token and length
  };
  auto group_item = [&](int G) {
    Item x;
    x.G = G;
    x.gi = 0;
    x.ci = G / p.Hk;
    x.hk = G - x.ci * p.Hk;
    x.h = x.hk * p.group;
    x.t0 = 0;
    x.L = 0;
    if (G < n_groups) {
      x.t0 = ws.ct.tok0[x.ci];
      x.L = ws.ct.len[x.ci];
    }
    return x;
  };
  auto next_item = [&](const Item& x) {
    if (x.gi + 1 < p.group) {
      Item y = x;
      ++y.gi;
      ++y.h;
      return y;
    }
    return group_item(x.G + int(gridDim.x));
  };

  if (w == 0) tc::tmem_alloc(&tmem_base, 512);
  if (tid == 0) {
    for (int b = 0; b < 5; ++b) tc::mbar_init(&bar[b], 1);
    for (int b = 0; b < 3; ++b) tc::mbar_init(&ldbar[b], 1);
    tc::fence_mbar_init();
  }
  // Phase-1 tiles of one (chunk, head) other than [K;Q], issued by thread 0 on ldbar[0]: the
  // workspace images and the per-token stats by bulk copy and the caller's v, dO rows by TMA (rows
  // past the sequence are zeroed after the wait).
  auto issue_phase1 = [&](const Item& x) {
    if (tid != 0) return;
    const int ci_ = x.ci, h_ = x.h;
    const int64_t ch_ = int64_t(ci_) * p.Hv + h_;
    const int t0_ = x.t0;
    tc::fence_proxy_async();
    tc::mbar_expect_tx(&ldbar[0], 2 * 8192 * 2 + 2 * 16384 * 2 + 2 * 16384 + 2048);
    tc::bulk_load(sm + lay::DVP, ws.dvp + ch_ * 8192, 16384, &ldbar[0]);
    tc::bulk_load(sm + lay::ST, ws.hs + ch_ * 16384, 32768, &ldbar[0]);
    tc::bulk_load(sm + lay::DHT, ws.dh + ch_ * 16384, 32768, &ldbar[0]);
    tc::bulk_load(sm + lay::VPT, ws.vp + ch_ * 8192, 16384, &ldbar[0]);
    tc::tma_rows128(sm + lay::VT, 8192, 0, &map_v, h_, t0_, &ldbar[0]);
    tc::tma_rows128(sm + lay::DOT, 8192, 0, &map_do, h_, t0_, &ldbar[0]);
    tc::bulk_load(sm + lay::STATS, ws.stats + ch_ * 512, 2048, &ldbar[0]);
  };
  // [K;Q] rows of one (chunk, key head) by TMA on ldbar[2]. The value heads of a group share them,
  // so they are fetched only when the (chunk, key head) changes, during the previous item's final
  // epilogue once its reads of the region are done.
  auto issue_kq = [&](const Item& x) {
    if (tid != 0) return;
    const int hk_ = x.hk;
    const int t0_ = x.t0;
    tc::fence_proxy_async();
    tc::mbar_expect_tx(&ldbar[2], 32768);
    tc::tma_rows128(sm + lay::KQ, 16384, 0, &map_k, hk_, t0_, &ldbar[2]);
    tc::tma_rows128(sm + lay::KQ, 16384, 64, &map_q, hk_, t0_, &ldbar[2]);
  };
  tc::fence_before_sync();
  __syncthreads();  // barrier init and the TMEM address visible
  tc::fence_after_sync();
  Item cur = group_item(int(blockIdx.x));
  if (cur.G < n_groups) {
    issue_phase1(cur);
    issue_kq(cur);
  }
  uint32_t kq_ph = 0;     // parity of the next [K;Q] load to wait for
  int prev_G = -1;        // the group whose [K;Q] rows are in shared memory
  const uint32_t tbase = tmem_base;
  const uint32_t lane_addr = tbase + (uint32_t(32 * q4) << 16) + c0;  // this thread's lane and column quarter
  const uint32_t kqa = tc::smem_u32(sm + lay::KQ);
  for (uint32_t it = 0; cur.G < n_groups; ++it) {
  const Item nxt = next_item(cur);
  const bool has_next = nxt.G < n_groups;
  const uint32_t ph = it & 1u;  // parity of the barriers that complete once per item
  const int ci = cur.ci, h = cur.h, hk = cur.hk;
  const int t0 = cur.t0, L = cur.L;
  const int64_t ch = int64_t(ci) * p.Hv + h;
  if (prev_G != cur.G) {  // issued at the start or by the previous item
    tc::mbar_wait(&ldbar[2], kq_ph, ws.err, 137);
    kq_ph ^= 1u;
  }
  prev_G = cur.G;
  tc::mbar_wait(&ldbar[0], ph, ws.err, 130);
  if (tid < 64) {
    const float* st = reinterpret_cast<const float*>(sm + lay::STATS);
    cum[tid] = st[tid]; rq[tid] = st[64 + tid]; rk[tid] = st[128 + tid]; beta[tid] = st[192 + tid];
    ecum[tid] = st[384 + tid];  // e^cum
    edec[tid] = st[448 + tid];  // e^(cum_last - cum)
    dbeta_acc[tid] = 0.f;
    dcum_acc[tid] = 0.f;
  }
  if (L < 64) {  // rows past the end of the sequence: zero (TMA fills only past the tensor's end)
    tc::zero_rows_tail(sm + lay::KQ, 16384, 0, L, kBThreads);
    tc::zero_rows_tail(sm + lay::KQ, 16384, 64, L, kBThreads);
    tc::zero_rows_tail(sm + lay::VT, 8192, 0, L, kBThreads);
    tc::zero_rows_tail(sm + lay::DOT, 8192, 0, L, kBThreads);
  }
  sync_for_mma();
  if (tid == 0) {  // ---- G1 ----
    // V'^T and dV'^T arrive as [dv][tok] tiles: read MN-major as the N = tok operand
    const uint64_t d_kq = tc::desc_kmajor_sw128(kqa), d_s = tc::desc_mnmajor_sw128(tc::smem_u32(sm + lay::ST), 16384),
                   d_dh = tc::desc_mnmajor_sw128(tc::smem_u32(sm + lay::DHT), 16384),
                   d_do = tc::desc_kmajor_sw128(tc::smem_u32(sm + lay::DOT)),
                   d_vp = tc::desc_mnmajor_sw128(tc::smem_u32(sm + lay::VPT), 8192),
                   d_dv = tc::desc_mnmajor_sw128(tc::smem_u32(sm + lay::DVP), 8192);
    const uint32_t id_kk = tc::idesc_bf16(128, 64, false, false);
    const uint32_t id_s = tc::idesc_bf16(128, 64, true, false);
    const uint32_t id_ss = tc::idesc_bf16(128, 64, true, true);
    const uint32_t id_sn = tc::idesc_bf16(128, 64, true, true, true);
    const uint32_t id_64 = tc::idesc_bf16(64, 64, false, true);
#pragma unroll 1  // issue loops stay rolled: the kernel is larger than the instruction cache
    for (int k0 = 0; k0 < 128; k0 += 16) {
      // descriptor address fields advance in 16-byte units: K-major by the k offset within the slab,
      // MN-major by k0 rows of 128 bytes
      const uint32_t o16 = ((k0 >> 6) * 16384 + (k0 & 63) * 2) >> 4, o8 = ((k0 >> 6) * 8192 + (k0 & 63) * 2) >> 4,
                     om = k0 * 8;
      const bool acc = k0 > 0;
      tc::mma_bf16(tbase + 0, d_kq + o16, d_kq + o16, id_kk, acc);
      tc::mma_bf16(tbase + 64, d_s + om, d_do + o8, id_s, acc);
      tc::mma_bf16(tbase + 128, d_s + om, d_dv + om, id_sn, acc);
      tc::mma_bf16(tbase + 192, d_dh + om, d_vp + om, id_ss, acc);
      tc::mma_bf16(tbase + 256, d_do + o8, d_vp + om, id_64, acc);
    }
    tc::mma_commit(&bar[0]);
  }
  {  // dgamma = sum S^T * dS^T while G1 runs (both tiles share one layout); warp 0 issues G1
    float part = 0.f;
    for (int idx = tid - 32; w > 0 && idx < 128 * 16; idx += kBThreads - 32) {
      const uint32_t off = uint32_t(idx) * 16;
      const uint4 a = *reinterpret_cast<const uint4*>(sm + lay::ST + off);
      const uint4 b = *reinterpret_cast<const uint4*>(sm + lay::DHT + off);
      const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) part += bf_lo(av[j]) * bf_lo(bv[j]) + bf_hi(av[j]) * bf_hi(bv[j]);
    }
    part = warp_sum(part);
    if (l == 0) red[w] = part;
  }
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int i = 0; i < kBThreads / 32; ++i) t += red[i];
    scal[0] = t;
  }
  tc::mbar_wait(&bar[0], ph, ws.err, 131);
  tc::fence_after_sync();
  if (tid == 0) {  // T (tile image) over dS^T, which G1 and the dgamma sum have consumed
    tc::fence_proxy_async();
    tc::mbar_expect_tx(&ldbar[1], 8192);
    tc::bulk_load(sm + lay::TT, ws.tinv + ch * 4096, 8192, &ldbar[1]);
  }
  // ---- E1 ------------------------------------------------------------------------------------
  {
    float v[16];
    tmem_ld16f(lane_addr + 0, v);  // lanes 0-63: kk rows, 64-127: qk rows
    float* dstf = r < 64 ? kkf + r * 65 + c0 : qkf + (r - 64) * 65 + c0;
#pragma unroll
    for (int j = 0; j < 16; ++j) dstf[j] = v[j];
    tmem_ld16f(lane_addr + 128, v);  // dW^T row dk = r
    store_row16(sm + lay::DWT, 128, r, c0, v);
    tmem_ld16f(lane_addr + 256, v);  // dA_qk (M = 64)
    if (mrow) {
#pragma unroll
      for (int j = 0; j < 16; ++j) daqf[i64 * 65 + c0 + j] = c0 + j <= i64 ? v[j] : 0.f;
    }
  }
  sync_for_mma();
  tc::mbar_wait(&ldbar[1], ph, ws.err, 136);
  const uint32_t tta = tc::smem_u32(sm + lay::TT), dwa = tc::smem_u32(sm + lay::DWT);
  if (tid == 0) {  // ---- G2 ----
    const uint32_t dva = tc::smem_u32(sm + lay::DVP);
    const uint64_t d_dvm = tc::desc_mnmajor_sw128(dva, 8192), d_dwm = tc::desc_mnmajor_sw128(dwa, 16384),
                   d_v = tc::desc_kmajor_sw128(tc::smem_u32(sm + lay::VT));
    const uint32_t id_t = tc::idesc_bf16(64, 64, true, false);
    // dT = dV' (beta V)^T + dW (beta e^cum r_k K)^T = (dV' V^T + dW K^T diag(e^cum r_k)) diag(beta): the two
    // products on the raw V and K rows, the per-token factors in E2's fp32 epilogue
#pragma unroll 4
    for (int k0 = 0; k0 < 128; k0 += 16)  // dV' V^T, dV' read MN-major from the dV'^T tile
      tc::mma_bf16(tbase + 320, d_dvm + k0 * 8, d_v + (((k0 >> 6) * 8192 + (k0 & 63) * 2) >> 4), id_t, k0 > 0);
#pragma unroll 4
    for (int k0 = 0; k0 < 128; k0 += 16)  // dW K^T, K = rows 0-63 of the [K;Q] tile
      tc::mma_bf16(tbase + 0, d_dwm + k0 * 8, tc::desc_kmajor_sw128(kqa) + (((k0 >> 6) * 16384 + (k0 & 63) * 2) >> 4), id_t,
                   k0 > 0);
    const uint64_t d_dvk = tc::desc_kmajor_sw128(dva), d_dwk = tc::desc_kmajor_sw128(dwa), d_t = tc::desc_mnmajor_sw128(tta, 8192);
    const uint32_t id_b = tc::idesc_bf16(128, 64, false, true);
#pragma unroll
    for (int k0 = 0; k0 < 64; k0 += 16) {  // dBv^T = dV'^T T, dBk^T = dW^T T
      tc::mma_bf16(tbase + 128, d_dvk + (k0 >> 3), d_t + k0 * 8, id_b, k0 > 0);
      tc::mma_bf16(tbase + 256, d_dwk + (k0 >> 3), d_t + k0 * 8, id_b, k0 > 0);
    }
    tc::mma_commit(&bar[1]);
  }
  tc::mbar_wait(&bar[1], ph, ws.err, 132);
  tc::fence_after_sync();
  // ---- E2 ------------------------------------------------------------------------------------
  {
    float v[16];
    tmem_ld16f(lane_addr + 320, v);  // dV' V^T (M = 64)
    {
      float z[16];
      tmem_ld16f(lane_addr + 0, z);  // dW K^T
      if (mrow) {  // dT[i][m] = beta_m (dV' V^T + e^cum_m r_k,m dW K^T)[i][m], lower triangle
#pragma unroll
        for (int j4 = 0; j4 < 16; j4 += 4) {
          const float4 b4 = *reinterpret_cast<const float4*>(beta + c0 + j4), e4 = *reinterpret_cast<const float4*>(ecum + c0 + j4),
                       k4 = *reinterpret_cast<const float4*>(rk + c0 + j4);
          const float bs[4] = {b4.x, b4.y, b4.z, b4.w}, es[4] = {e4.x, e4.y, e4.z, e4.w}, ks[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = j4 + u;
            v[j] = c0 + j <= i64 ? bs[u] * fmaf(es[u] * ks[u], z[j], v[j]) : 0.f;
          }
        }
        store_row16(sm + lay::DTT, 64, i64, c0, v);
      }
    }
    tmem_ld16f(lane_addr + 128, v);  // dBv^T row dv = r, columns m = c0 + j
    float x[16], bt[16];
    lds_vec(beta + c0, bt);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      x[j] = bt[j] * v[j];
      v[j] *= tile_elem(sm + lay::VT, 64, c0 + j, r);
    }
    // dv rows are staged over dW^T (dead after G2) and written out after the last proxy fence
    stage_cols16(reinterpret_cast<bf16*>(sm + lay::DVS), r, c0, x);
    const float cs = warp_colsum16(v);
    if ((l & 1) == 0) red[q4 * 64 + c0 + (l >> 1)] = cs;
  }
  __syncthreads();
  if (tid < 64) dbeta_acc[tid] += red[tid] + red[64 + tid] + red[128 + tid] + red[192 + tid];
  sync_for_mma();
  if (tid == 0) {  // ---- G3: Y = T^T dT ----
    const uint64_t d_t = tc::desc_mnmajor_sw128(tta, 8192), d_dt = tc::desc_mnmajor_sw128(tc::smem_u32(sm + lay::DTT), 8192);
    const uint32_t id_y = tc::idesc_bf16(64, 64, true, true);
#pragma unroll
    for (int k0 = 0; k0 < 64; k0 += 16) tc::mma_bf16(tbase + 0, d_t + k0 * 8, d_dt + k0 * 8, id_y, k0 > 0);
    tc::mma_commit(&bar[2]);
  }
  tc::mbar_wait(&bar[2], ph, ws.err, 133);
  tc::fence_after_sync();
  {
    float v[16];
    tmem_ld16f(lane_addr + 0, v);
    if (mrow) {  // [Y; Y]: G4 runs with M = 128 so that E4 has a row in every lane
      store_row16(sm + lay::YT, 128, i64, c0, v);
      store_row16(sm + lay::YT, 128, 64 + i64, c0, v);
    }
  }
  sync_for_mma();
  if (tid == 0) {  // ---- G4: dL' = Y T^T ----
    const uint64_t d_y = tc::desc_kmajor_sw128(tc::smem_u32(sm + lay::YT)), d_t = tc::desc_kmajor_sw128(tta);
    const uint32_t id_l = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
    for (int k0 = 0; k0 < 64; k0 += 16) tc::mma_bf16(tbase + 128, d_y + (k0 >> 3), d_t + (k0 >> 3), id_l, k0 > 0);
    tc::mma_commit(&bar[3]);
  }
  tc::mbar_wait(&bar[3], ph, ws.err, 134);
  tc::fence_after_sync();
  // ---- E4: P, Qm, R and the B operands of G5. dL' is an M = 128 accumulator of [Y; Y] T^T, so
  // lane 32 q4 + l holds token row i = (32 q4 + l) & 63; the thread takes 8 columns, cb..cb+7.
  {
    const int i = r & 63, cb = c0 + 8 * (q4 >> 1);
    float v[8];
    tc::tmem_ld8(tbase + (uint32_t(32 * q4) << 16) + 128 + cb, v);
    const float bi = beta[i], rki = rk[i], sqi = p.scale * rq[i], ci_ = cum[i];
    float db = 0.f;
    float pb1[8], qb1[8], pb2[8], qb2[8];
    float cj[8], rkj[8], ex[8];  // the columns' cum and r_k (16-byte loads) and e^(c_i - c_j), all first
    *reinterpret_cast<float4*>(cj) = *reinterpret_cast<const float4*>(cum + cb);
    *reinterpret_cast<float4*>(cj + 4) = *reinterpret_cast<const float4*>(cum + cb + 4);
    *reinterpret_cast<float4*>(rkj) = *reinterpret_cast<const float4*>(rk + cb);
    *reinterpret_cast<float4*>(rkj + 4) = *reinterpret_cast<const float4*>(rk + cb + 4);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) ex[jj] = __expf(ci_ - cj[jj]);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int j = cb + jj;
      const float gam = j <= i ? ex[jj] : 0.f;
      const float P = j < i ? -v[jj] * gam : 0.f;
      const float kkn = kkf[i * 65 + j] * rki * rkj[jj];
      const float qkn = qkf[i * 65 + j] * sqi * rkj[jj];
      const float daq = daqf[i * 65 + j];
      const float qm = daq * gam;
      db = fmaf(P, kkn, db);
      kkf[i * 65 + j] = P * bi * kkn + daq * qkn * gam;  // R
      pb1[jj] = bi * rkj[jj] * P;
      qb1[jj] = rkj[jj] * qm;
      pb2[jj] = bi * rki * P;
      qb2[jj] = sqi * qm;
    }
    dbp[(2 * cq + (q4 >> 1)) * 64 + i] = db;
    store_row8(sm + lay::PB1, 64, i, cb, pb1);
    store_row8(sm + lay::QB1, 64, i, cb, qb1);
    store_row8(sm + lay::PB2, 64, i, cb, pb2);
    store_row8(sm + lay::QB2, 64, i, cb, qb2);
  }
  sync_for_mma();
  // dv rows of the chunk: coalesced 16-byte stores by warps 8-15 while G5 runs
  copy_rows_out(dv + (int64_t(t0) * p.Hv + h) * 128, int64_t(p.Hv) * 256, sm + lay::DVS, 256, L, kBThreads / 2,
                kBThreads / 2);
  if (tid == 0) {  // ---- G5 ----
    const uint64_t d_k = tc::desc_mnmajor_sw128(kqa, 16384),         // K rows as (M = dk, K = j)
        d_q = tc::desc_mnmajor_sw128(kqa + 8192, 16384),              // Q rows (start at row 64)
        d_p1 = tc::desc_kmajor_sw128(tc::smem_u32(sm + lay::PB1)), d_q1 = tc::desc_kmajor_sw128(tc::smem_u32(sm + lay::QB1)),
                   d_p2 = tc::desc_mnmajor_sw128(tc::smem_u32(sm + lay::PB2), 8192),
                   d_q2 = tc::desc_mnmajor_sw128(tc::smem_u32(sm + lay::QB2), 8192);
    const uint32_t id_k = tc::idesc_bf16(128, 64, true, false), id_m = tc::idesc_bf16(128, 64, true, true);
#pragma unroll 1  // issue loops stay rolled: the kernel is larger than the instruction cache
    for (int k0 = 0; k0 < 64; k0 += 16) {
      const uint32_t om = k0 * 8, ok = k0 >> 3;
      tc::mma_bf16(tbase + 320, d_k + om, d_p1 + ok, id_k, k0 > 0);
      tc::mma_bf16(tbase + 320, d_k + om, d_p2 + om, id_m, true);
      tc::mma_bf16(tbase + 320, d_q + om, d_q2 + om, id_m, true);
      tc::mma_bf16(tbase + 0, d_k + om, d_q1 + ok, id_k, k0 > 0);
    }
    tc::mma_commit(&bar[4]);
  }
  constexpr int kParts = (kBThreads - 64) / 64;  // dcum row / column sums split over warps 2..15
  if (tid >= 64) {  // dcum_i += sum_j R_ij - sum_j R_ji, in kParts ranges of j (warp 0 issues G5)
    const int i = (tid - 64) & 63, part = (tid - 64) >> 6;
    const int j0 = (64 * part) / kParts, j1 = (64 * (part + 1)) / kParts;
    float a = 0.f;
    for (int j = j0; j < j1; ++j) a += kkf[i * 65 + j] - kkf[j * 65 + i];
    daqf[part * 64 + i] = a;  // dA_qk (E4's input) is dead
    if (part == 0) {
      float d = 0.f;
#pragma unroll
      for (int b = 0; b < 8; ++b) d += dbp[b * 64 + i];
      dbeta_acc[i] += d;
    }
  }
  tc::mbar_wait(&bar[4], ph, ws.err, 135);
  tc::fence_after_sync();
  __syncthreads();  // region A (the phase-2 tiles) is free once G5 has completed
  if (has_next) issue_phase1(nxt);  // next item's tiles, behind this epilogue
  if (tid < 64) {
    float a = 0.f;
#pragma unroll
    for (int b = 0; b < kParts; ++b) a += daqf[b * 64 + tid];
    dcum_acc[tid] += a;
  }
  // ---- final epilogue: thread = head-dim row r, tokens i = c0 + j; q[i][r], k[i][r] read from the
  // [K;Q] tile (consecutive lanes read consecutive columns of one row: no bank conflicts) -----------
  float xr[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) xr[j] = tile_elem(sm + lay::KQ, 128, 64 + c0 + j, r);
  float* red1 = red;            // a1: sum_r dq~^T q
  float* red2 = red + 256;      // a4: sum_r dq^^T q   (l2norm)
  float* red3 = red + 512;      // a2: sum_r dk~^T k
  float* red4 = red + 768;      // a3: sum_r dBk^T k
  float* red5 = red + 1024;     // a5: sum_r dk^^T k   (l2norm)
  const int rslot = q4 * 64 + c0 + (l >> 1);  // this lane's column of a warp_colsum16 (even lanes write it)
  const bool wr = (l & 1) == 0;
  float dqh[16];
  {
    float t1[16], v[16], ec[16];
    tmem_ld16f(lane_addr + 0, dqh);   // (Qm k^)^T
    tmem_ld16f(lane_addr + 64, t1);   // dq~^T
    lds_vec(ecum + c0, ec);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      dqh[j] = p.scale * fmaf(ec[j], t1[j], dqh[j]);
      v[j] = t1[j] * xr[j];
      t1[j] = dqh[j] * xr[j];
    }
    const float s1 = warp_colsum16(v), s2 = warp_colsum16(t1);
    if (wr) { red1[rslot] = s1; red2[rslot] = s2; }
  }
  float kr_[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) kr_[j] = tile_elem(sm + lay::KQ, 128, c0 + j, r);
  float dkh[16];
  {
    float t2[16], t3[16], ed[16], bt[16], ec[16];
    tmem_ld16f(lane_addr + 320, dkh);  // diag(beta) P k^ + P^T diag(beta) k^ + Qm^T q^   (transposed)
    tmem_ld16f(lane_addr + 192, t2);   // dk~^T
    tmem_ld16f(lane_addr + 256, t3);   // dBk^T
    lds_vec(edec + c0, ed);
    lds_vec(beta + c0, bt);
    lds_vec(ecum + c0, ec);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      dkh[j] = fmaf(ed[j], t2[j], fmaf(bt[j] * ec[j], t3[j], dkh[j]));
      t2[j] *= kr_[j];
      t3[j] *= kr_[j];
    }
    const float s3 = warp_colsum16(t2), s4 = warp_colsum16(t3);
#pragma unroll
    for (int j = 0; j < 16; ++j) t2[j] = dkh[j] * kr_[j];
    const float s5 = warp_colsum16(t2);
    if (wr) { red3[rslot] = s3; red4[rslot] = s4; red5[rslot] = s5; }
  }
  __syncthreads();  // every thread holds its q and k rows (xr, kr_): [K;Q] may be refilled
  {
    if (has_next && nxt.G != cur.G) issue_kq(nxt);
  }
  if (tid < 64) {  // combine the four lane quarters
#pragma unroll
    for (int b = 0; b < 5; ++b) {
      float* rb = red + 256 * b;
      rb[tid] = rb[tid] + rb[64 + tid] + rb[128 + tid] + rb[192 + tid];
    }
  }
  __syncthreads();
  {
    float gq[16], gk[16];
    {
      float rqv[16], rkv[16], a4[16], a5[16];
      lds_vec(rq + c0, rqv);
      lds_vec(rk + c0, rkv);
      lds_vec(red2 + c0, a4);
      lds_vec(red5 + c0, a5);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float rqi = rqv[j], rki = rkv[j];
        gq[j] = rqi * dqh[j] - xr[j] * rqi * rqi * rqi * a4[j];
        gk[j] = rki * dkh[j] - kr_[j] * rki * rki * rki * a5[j];
      }
    }
    bool last = true;  // this value head completes dq / dk of its key head
    if (p.group > 1) {  // GQA: the group's running sum in fp32, kept in TMEM columns [384, 512) until its last value head
      if (cur.gi > 0) {
        float pq[16];
        tmem_ld16f(lane_addr + 384, pq);
#pragma unroll
        for (int j = 0; j < 16; ++j) gq[j] += pq[j];
        tmem_ld16f(lane_addr + 448, pq);
#pragma unroll
        for (int j = 0; j < 16; ++j) gk[j] += pq[j];
      }
      if (cur.gi + 1 < p.group) {
        tc::tmem_st16(lane_addr + 384, gq);
        tc::tmem_st16(lane_addr + 448, gk);
        last = false;
      }
    }
    if (last) {
      const int row = p.Hk * 128;
      store_cols16(dq + (int64_t(t0) * p.Hk + hk) * 128, row, r, c0, L, gq);
      store_cols16(dk + (int64_t(t0) * p.Hk + hk) * 128, row, r, c0, L, gk);
    }
  }
  // ---- per-token scalars: dcum, dbeta, dg -----------------------------------------------------
  if (tid < 64) {
    const int i = tid;
    const float z = edec[i] * rk[i] * red3[i];
    const float colk = rk[i] * red4[i];
    dcum_acc[i] += ecum[i] * p.scale * rq[i] * red1[i] - z + beta[i] * ecum[i] * colk;
    dbeta_acc[i] += ecum[i] * colk;
    scal[1 + i] = z;
  }
  __syncthreads();
  if (w == 0) {  // dg = reverse cumulative sum of dcum (in double), lane l: tokens l and 32 + l
    const float dcl = scal[0] * expf(cum[63]) + warp_sum(scal[1 + l] + scal[33 + l]);
    double lo = dcum_acc[l], hi = l == 31 ? double(dcum_acc[63] + dcl) : double(dcum_acc[32 + l]);
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const double tl = __shfl_down_sync(0xffffffffu, lo, off), th = __shfl_down_sync(0xffffffffu, hi, off);
      if (l + off < 32) { lo += tl; hi += th; }
    }
    lo += __shfl_sync(0xffffffffu, hi, 0);
    if (l < L) dg[int64_t(t0 + l) * p.Hv + h] = float(lo);
    if (32 + l < L) dg[int64_t(t0 + 32 + l) * p.Hv + h] = float(hi);
  }
  if (tid < L && tid < 64) dbeta[int64_t(t0 + tid) * p.Hv + h] = __float2bfloat16_rn(dbeta_acc[tid]);
  tc::fence_before_sync();
  __syncthreads();  // this item's TMEM and shared reads are done before the next item's MMAs and loads
  cur = nxt;
  }
  if (w == 0) tc::tmem_dealloc(tbase, 512);
}


template <typename K>
int smem_attr_b(K kernel, int bytes) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return RB2_ECUDA;
  }
  return RB2_OK;
}

}  // namespace

int fast_backward(const GdnProblem& p, void* wsp, void* scratch, const void* d_o, const float* dhT, void* dq, void* dk,
                  void* dv, float* dg, void* dbeta, float* dh0, cudaStream_t s) {
  Carver c(wsp);
  FastWs w;
  const size_t saved = carve_fast_saved(c, w, p.n_seqs, p.Hv, p.max_chunks);
  Carver c2(scratch ? scratch : static_cast<char*>(wsp) + saved);
  carve_fast_scratch(c2, w, p.tokens, p.Hv, p.max_chunks, p.group > 1);
  int rc;
  if ((p.stages & 1) && (rc = smem_attr_b(fast_state_bwd_kernel, kBStateSmem))) return rc;
  if (p.stages & 1) {
    ProfScope ps_("gdn_fast_state_bwd", s);
    CUtensorMap mdo;
    if ((rc = make_rows_map(&mdo, d_o, p.tokens, p.Hv))) return rc;
    CUtensorMap mk;
    if ((rc = make_rows_map(&mk, p.k, p.tokens, p.Hk))) return rc;
    fast_state_bwd_kernel<<<dim3(p.Hv, unsigned(p.n_seqs)), 256, kBStateSmem, s>>>(p, w, mdo, dhT, dh0, mk);
    RB2_CHECK_LAUNCH("gdn fast state bwd");
  }
  if ((p.stages & 2) && p.max_chunks > 0) {
    if ((rc = smem_attr_b(fast_chunk_bwd_kernel, kBChunkSmem))) return rc;
    {
      ProfScope ps_("gdn_fast_chunk_bwd", s);
      int dev = 0, sms = 148;
      RB2_CUDA(cudaGetDevice(&dev), "gdn fast chunk bwd: device");
      RB2_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "gdn fast chunk bwd: SM count");
      const int64_t items = int64_t(p.max_chunks) * p.Hk;  // (chunk, key head) groups
      RB2_CHECK_ARG(items + sms < (int64_t(1) << 31), "gdn fast chunk bwd: %lld (chunk, key head) groups exceed 2^31",
                    (long long)items);
      CUtensorMap mq, mk, mv, mdo;
      if ((rc = make_rows_map(&mq, p.q, p.tokens, p.Hk)) || (rc = make_rows_map(&mk, p.k, p.tokens, p.Hk)) ||
          (rc = make_rows_map(&mv, p.v, p.tokens, p.Hv)) || (rc = make_rows_map(&mdo, d_o, p.tokens, p.Hv)))
        return rc;
      fast_chunk_bwd_kernel<<<unsigned(items < sms ? items : sms), kBThreads, kBChunkSmem, s>>>(
          p, w, static_cast<const bf16*>(d_o), static_cast<bf16*>(dq), static_cast<bf16*>(dk), static_cast<bf16*>(dv), dg,
          static_cast<bf16*>(dbeta), mq, mk, mv, mdo);
      RB2_CHECK_LAUNCH("gdn fast chunk bwd");
    }
  }
  return RB2_OK;
}

}  // namespace rb2
