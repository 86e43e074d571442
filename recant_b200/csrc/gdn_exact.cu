// Chunked Gated DeltaNet, exact path: fp32 CUDA-core arithmetic throughout.
//
// This is the fp32-parity path (rel. Frobenius <= 1e-4 against recant.model.ops.gdn_torch,
// recant/model/ops.py:21-54, and its autograd backward). It follows the same chunked
// factorisation as the reference so that underflowing decays behave identically:
//   Gamma_ij = exp(cum_i - cum_j) (i >= j), q~ = q e^cum, k~ = k e^(cum_last - cum).
// cum is accumulated in double and rounded once per element, which is how torch's CPU cumsum
// (used by ops.py:36) computes a float32 prefix sum, so cum is bit-identical to the reference.
//
// Kernels (one CTA = 256 threads; "ch" = (chunk, value head)):
//   fwd_prep   per ch      : l2norm, cum, A_kk, A_qk, T = (I + A_kk)^-1, U = T beta V,
//                            W = T beta e^cum K
//   fwd_state  per (seq, head, 32 state columns): S walk over the chunks, V' = U - W S,
//                            S <- gamma S + k~^T V'
//   fwd_out    per ch      : O = q~ S + A_qk V'
//   bwd_state  per (seq, head, 32 columns): reversed dS walk,
//                            dV' = A_qk^T dO + k~ dS,  dS <- gamma dS + q~^T dO - W^T dV'
//   bwd_mm     per ch      : dq~ = dO S^T, dW = -dV' S^T, dk~ = V' dS_next^T, dA_qk, dgamma
//   bwd_intra  per ch      : back through T, the masks, the decays and the l2norm
//   bwd_gqa    per token   : sums per-value-head dq/dk over each key-head group
#include "gdn_common.cuh"

namespace rb2 {
namespace {

constexpr int kThreads = 256;

// Register fragment of an M x N fp32 tile spread over 256 threads: warp w owns rows
// w + 8*ii, lane l owns columns l + 32*jj.
template <int M, int N>
struct Frag {
  static_assert(M % 8 == 0 && N % 32 == 0, "fragment shape");
  float v[M / 8][N / 32];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < M / 8; ++i)
#pragma unroll
      for (int j = 0; j < N / 32; ++j) v[i][j] = 0.f;
  }
};

__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

// acc += A . B with A(i,k) = A[i*a_rs + k*a_cs] (rows >= m_valid or k >= k_valid read as 0)
// and B(k,j) = B[k*b_rs + j*b_cs] (k >= k_valid read as 0). K is streamed 16 at a time
// through shared memory (sA: M x 17 floats, sB: 16 x (N+1) floats). All threads must call.
template <int M, int N, typename TA, typename TB>
__device__ void block_mm(Frag<M, N>& acc, const TA* A, int64_t a_rs, int64_t a_cs, int m_valid,
                         const TB* B, int64_t b_rs, int64_t b_cs, int K, int k_valid,
                         float* sA, float* sB) {
  for (int k0 = 0; k0 < K; k0 += 16) {
    if (a_cs == 1) {
      for (int idx = threadIdx.x; idx < M * 16; idx += kThreads) {
        const int i = idx >> 4, kk = idx & 15, k = k0 + kk;
        sA[i * 17 + kk] = (i < m_valid && k < k_valid) ? ldf(A + i * a_rs + k) : 0.f;
      }
    } else {
      for (int idx = threadIdx.x; idx < M * 16; idx += kThreads) {
        const int i = idx % M, kk = idx / M, k = k0 + kk;
        sA[i * 17 + kk] = (i < m_valid && k < k_valid) ? ldf(A + i * a_rs + k * a_cs) : 0.f;
      }
    }
    if (b_cs == 1) {
      for (int idx = threadIdx.x; idx < 16 * N; idx += kThreads) {
        const int kk = idx / N, j = idx % N, k = k0 + kk;
        sB[kk * (N + 1) + j] = (k < k_valid) ? ldf(B + k * b_rs + j) : 0.f;
      }
    } else {
      for (int idx = threadIdx.x; idx < 16 * N; idx += kThreads) {
        const int kk = idx & 15, j = idx >> 4, k = k0 + kk;
        sB[kk * (N + 1) + j] = (k < k_valid) ? ldf(B + k * b_rs + j * b_cs) : 0.f;
      }
    }
    __syncthreads();
    const int w = warp_id(), l = lane_id();
#pragma unroll 4
    for (int kk = 0; kk < 16; ++kk) {
      float a[M / 8], b[N / 32];
#pragma unroll
      for (int i = 0; i < M / 8; ++i) a[i] = sA[(w + 8 * i) * 17 + kk];
#pragma unroll
      for (int j = 0; j < N / 32; ++j) b[j] = sB[kk * (N + 1) + l + 32 * j];
#pragma unroll
      for (int i = 0; i < M / 8; ++i)
#pragma unroll
        for (int j = 0; j < N / 32; ++j) acc.v[i][j] = fmaf(a[i], b[j], acc.v[i][j]);
    }
    __syncthreads();
  }
}

// Sum over all threads of the block (result valid in every thread). `red` holds 8 floats.
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if (lane_id() == 0) red[warp_id()] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) t += red[i];
  __syncthreads();
  return t;
}

__global__ void chunk_table_kernel(const int64_t* __restrict__ cu, int64_t n_seqs, int64_t T,
                                   int max_chunks, ChunkTable ct) {
  __shared__ int scan[1024];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < n_seqs; base += 1024) {
    const int64_t i = base + threadIdx.x;
    int64_t s0 = 0, L = 0;
    if (i < n_seqs) {
      s0 = cu ? cu[i] : i * T;
      L = cu ? cu[i + 1] - cu[i] : T;
      if (L < 0) L = 0;
    }
    const int nch = int((L + kChunk - 1) / kChunk);
    scan[threadIdx.x] = nch;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {  // inclusive Hillis-Steele scan
      const int t = threadIdx.x >= off ? scan[threadIdx.x - off] : 0;
      __syncthreads();
      scan[threadIdx.x] += t;
      __syncthreads();
    }
    const int first = carry + scan[threadIdx.x] - nch;
    if (i < n_seqs) {
      ct.seq_chunk0[i] = first;
      for (int c = 0; c < nch; ++c) {
        const int idx = first + c;
        if (idx < max_chunks) {
          ct.tok0[idx] = int(s0 + int64_t(c) * kChunk);
          ct.len[idx] = int(L - int64_t(c) * kChunk < kChunk ? L - int64_t(c) * kChunk : kChunk);
          ct.seq[idx] = int(i);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 1023) carry += scan[1023];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    ct.seq_chunk0[n_seqs] = carry;
    *ct.n_chunks = carry;
  }
  // The walks' order of the sequences: longest first (ties: lower index), so that the CTAs of the
  // long ones start in the first wave and a short one, not a long one, finishes last (packs of up to
  // 1024 sequences, ranked from shared memory; larger packs and equal lengths keep the given order).
  __shared__ int len_s[1024];
  const bool rank_them = cu != nullptr && n_seqs <= 1024;
  for (int64_t i = threadIdx.x; i < n_seqs; i += 1024) {
    if (!rank_them) {
      ct.order[i] = int(i);
      continue;
    }
    len_s[i] = int(cu[i + 1] - cu[i]);
  }
  __syncthreads();
  if (rank_them && int64_t(threadIdx.x) < n_seqs) {
    const int i = int(threadIdx.x), li = len_s[i];
    int rank = 0;
    for (int j = 0; j < int(n_seqs); ++j) {
      const int lj = len_s[j];
      rank += (lj > li || (lj == li && j < i)) ? 1 : 0;
    }
    ct.order[rank] = i;
  }
  // entries past the last chunk read as empty (len 0): a kernel launched over max_chunks can skip
  // its chunk from its own entry, without first reading n_chunks
  for (int idx = carry + int(threadIdx.x); idx < max_chunks; idx += 1024) {
    ct.tok0[idx] = 0;
    ct.len[idx] = 0;
    ct.seq[idx] = 0;
  }
}

// ------------------------------------------------------------------------------------------
// forward
// ------------------------------------------------------------------------------------------
struct PrepSmem {
  float qn[64 * 129];
  float kn[64 * 129];
  float lm[64 * 65];
  float tm[64 * 65];
  float sA[64 * 17];
  float sB[16 * 129];
  float g[64], cum[64], ecum[64], beta[64], rq[64], rk[64];
};

// Rows of q or k for one chunk: normalised (times `mul`) into smem, row scale into r[].
template <typename TIn>
__device__ void load_normalised(const TIn* __restrict__ src, int64_t row_stride, int L, float mul,
                                float* dst, float* r) {
  for (int idx = threadIdx.x; idx < 64 * 128; idx += kThreads) {
    const int i = idx >> 7, c = idx & 127;
    dst[i * 129 + c] = i < L ? ldf(src + i * row_stride + c) : 0.f;
  }
  __syncthreads();
  const int w = warp_id(), l = lane_id();
  for (int i = w; i < 64; i += 8) {
    float s = 0.f;
#pragma unroll
    for (int m = 0; m < 4; ++m) { const float x = dst[i * 129 + l + 32 * m]; s = fmaf(x, x, s); }
    s = warp_sum(s);
    const float rs = 1.0f / sqrtf(s + 1e-6f);
    if (l == 0) r[i] = rs;
#pragma unroll
    for (int m = 0; m < 4; ++m) dst[i * 129 + l + 32 * m] = dst[i * 129 + l + 32 * m] * rs * mul;
  }
  __syncthreads();
}

// (I + L)^-1 for strictly-lower L (64x64, smem stride 65) into T (stride 65): the four 16x16
// diagonal blocks by forward substitution (one warp each, lane = column), then the
// off-diagonal blocks by block rows: T_ij = -T_ii sum_{j<=m<i} L_im T_mj.
__device__ void unit_lower_inverse(const float* lm, float* tm) {
  const int w = warp_id(), l = lane_id();
  for (int idx = threadIdx.x; idx < 64 * 65; idx += kThreads) tm[idx] = 0.f;
  __syncthreads();
  if (w < 4 && l < 16) {
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
  __syncthreads();
  __shared__ float xbuf[3 * 256];
  const int r = threadIdx.x >> 4, c = threadIdx.x & 15;
  for (int bi = 1; bi < 4; ++bi) {
    for (int bj = 0; bj < bi; ++bj) {  // X_bj = sum_{m = 16bj}^{16bi - 1} L[16bi + r][m] T[m][16bj + c]
      float x = 0.f;
      for (int m = 16 * bj; m < 16 * bi; ++m) x = fmaf(lm[(16 * bi + r) * 65 + m], tm[m * 65 + 16 * bj + c], x);
      xbuf[bj * 256 + r * 16 + c] = x;
    }
    __syncthreads();
    for (int bj = 0; bj < bi; ++bj) {
      float t = 0.f;
      for (int m = 0; m < 16; ++m) t = fmaf(tm[(16 * bi + r) * 65 + 16 * bi + m], xbuf[bj * 256 + m * 16 + c], t);
      tm[(16 * bi + r) * 65 + 16 * bj + c] = -t;
    }
    __syncthreads();
  }
}

template <typename TIn>
__global__ void __launch_bounds__(kThreads)
fwd_prep_kernel(GdnProblem p, ExactWs ws) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(smem_raw);
  const int ci = blockIdx.x, h = blockIdx.y;
  if (ci >= *ws.ct.n_chunks) return;
  const int t0 = ws.ct.tok0[ci], L = ws.ct.len[ci], hk = h / p.group;
  const int64_t ch = int64_t(ci) * p.Hv + h;
  const TIn* q = static_cast<const TIn*>(p.q) + (int64_t(t0) * p.Hk + hk) * 128;
  const TIn* k = static_cast<const TIn*>(p.k) + (int64_t(t0) * p.Hk + hk) * 128;
  const TIn* v = static_cast<const TIn*>(p.v) + (int64_t(t0) * p.Hv + h) * 128;
  const TIn* beta = static_cast<const TIn*>(p.beta);

  if (threadIdx.x < 64) {
    const int i = threadIdx.x;
    sm.g[i] = i < L ? p.g[int64_t(t0 + i) * p.Hv + h] : 0.f;
    sm.beta[i] = i < L ? ldf(beta + int64_t(t0 + i) * p.Hv + h) : 0.f;
  }
  load_normalised<TIn>(q, int64_t(p.Hk) * 128, L, p.scale, sm.qn, sm.rq);
  load_normalised<TIn>(k, int64_t(p.Hk) * 128, L, 1.f, sm.kn, sm.rk);
  if (threadIdx.x == 0) {
    double acc = 0.0;
    for (int i = 0; i < 64; ++i) { acc += double(sm.g[i]); sm.cum[i] = float(acc); }
  }
  __syncthreads();
  if (threadIdx.x < 64) sm.ecum[threadIdx.x] = expf(sm.cum[threadIdx.x]);
  float* st = ws.stats + ch * 256;
  if (threadIdx.x < 64) {
    const int i = threadIdx.x;
    st[i] = sm.cum[i]; st[64 + i] = sm.rq[i]; st[128 + i] = sm.rk[i]; st[192 + i] = sm.beta[i];
  }
  for (int idx = threadIdx.x; idx < 64 * 128; idx += kThreads) {
    const int i = idx >> 7, c = idx & 127;
    ws.qn[ch * 8192 + idx] = sm.qn[i * 129 + c];
    ws.kn[ch * 8192 + idx] = sm.kn[i * 129 + c];
  }
  __syncthreads();

  const int w = warp_id(), l = lane_id();
  {
    Frag<64, 64> kk, qk;
    kk.zero(); qk.zero();
    block_mm<64, 64>(kk, sm.kn, 129, 1, 64, sm.kn, 1, 129, 128, 128, sm.sA, sm.sB);
    block_mm<64, 64>(qk, sm.qn, 129, 1, 64, sm.kn, 1, 129, 128, 128, sm.sA, sm.sB);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int i = w + 8 * ii, j = l + 32 * jj;
        const float gam = j <= i ? expf(sm.cum[i] - sm.cum[j]) : 0.f;
        sm.lm[i * 65 + j] = j < i ? sm.beta[i] * kk.v[ii][jj] * gam : 0.f;
        ws.aqk[ch * 4096 + i * 64 + j] = j <= i ? qk.v[ii][jj] * gam : 0.f;
      }
    }
  }
  __syncthreads();
  unit_lower_inverse(sm.lm, sm.tm);
  for (int idx = threadIdx.x; idx < 64 * 64; idx += kThreads) {
    const int i = idx >> 6, j = idx & 63;
    const float t = sm.tm[i * 65 + j];
    ws.tinv[ch * 4096 + idx] = t;
    sm.lm[i * 65 + j] = t * sm.beta[j];  // T diag(beta)
  }
  __syncthreads();
  {
    Frag<64, 128> u;
    u.zero();
    block_mm<64, 128>(u, sm.lm, 65, 1, 64, v, int64_t(p.Hv) * 128, 1, 64, L, sm.sA, sm.sB);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) ws.u[ch * 8192 + (w + 8 * ii) * 128 + l + 32 * jj] = u.v[ii][jj];
  }
  for (int idx = threadIdx.x; idx < 64 * 64; idx += kThreads) {
    const int i = idx >> 6, j = idx & 63;
    sm.lm[i * 65 + j] = sm.tm[i * 65 + j] * (sm.beta[j] * sm.ecum[j]);  // T diag(beta e^cum)
  }
  __syncthreads();
  {
    Frag<64, 128> wf;
    wf.zero();
    block_mm<64, 128>(wf, sm.lm, 65, 1, 64, sm.kn, 129, 1, 64, 64, sm.sA, sm.sB);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) ws.w[ch * 8192 + (w + 8 * ii) * 128 + l + 32 * jj] = wf.v[ii][jj];
  }
}

struct StateSmem {
  float ss[128 * 33];
  float vs[64 * 33];
  float xs[64 * 33];
  float sA[128 * 17];
  float sB[16 * 33];
  float cum[64];
};

__global__ void __launch_bounds__(kThreads)
fwd_state_kernel(GdnProblem p, ExactWs ws, float* __restrict__ hT) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  StateSmem& sm = *reinterpret_cast<StateSmem*>(smem_raw);
  const int h = blockIdx.x, s = blockIdx.y, j0 = blockIdx.z * 32;
  const int w = warp_id(), l = lane_id();
  Frag<128, 32> S;
  const int64_t sbase = (int64_t(s) * p.Hv + h) * 16384;
#pragma unroll
  for (int ii = 0; ii < 16; ++ii) S.v[ii][0] = p.h0 ? p.h0[sbase + (w + 8 * ii) * 128 + j0 + l] : 0.f;
  const int c0 = ws.ct.seq_chunk0[s], c1 = ws.ct.seq_chunk0[s + 1];
  for (int ci = c0; ci < c1; ++ci) {
    const int64_t ch = int64_t(ci) * p.Hv + h;
#pragma unroll
    for (int ii = 0; ii < 16; ++ii) {
      const int r = w + 8 * ii;
      ws.hs[ch * 16384 + r * 128 + j0 + l] = S.v[ii][0];
      sm.ss[r * 33 + l] = S.v[ii][0];
    }
    if (threadIdx.x < 64) sm.cum[threadIdx.x] = ws.stats[ch * 256 + threadIdx.x];
    __syncthreads();
    Frag<64, 32> vp;
    vp.zero();
    block_mm<64, 32>(vp, ws.w + ch * 8192, 128, 1, 64, sm.ss, 33, 1, 128, 128, sm.sA, sm.sB);
    const float cl = sm.cum[63];
#pragma unroll
    for (int ii = 0; ii < 8; ++ii) {
      const int i = w + 8 * ii;
      const float x = ws.u[ch * 8192 + i * 128 + j0 + l] - vp.v[ii][0];
      ws.vp[ch * 8192 + i * 128 + j0 + l] = x;
      sm.vs[i * 33 + l] = x * expf(cl - sm.cum[i]);
    }
    __syncthreads();
    Frag<128, 32> upd;
    upd.zero();
    block_mm<128, 32>(upd, ws.kn + ch * 8192, 1, 128, 128, sm.vs, 33, 1, 64, 64, sm.sA, sm.sB);
    const float gamma = expf(cl);
#pragma unroll
    for (int ii = 0; ii < 16; ++ii) S.v[ii][0] = gamma * S.v[ii][0] + upd.v[ii][0];
    __syncthreads();
  }
  if (hT) {
#pragma unroll
    for (int ii = 0; ii < 16; ++ii) hT[sbase + (w + 8 * ii) * 128 + j0 + l] = S.v[ii][0];
  }
}

struct OutSmem {
  float sA[64 * 17];
  float sB[16 * 129];
  float cum[64];
};

template <typename TIn>
__global__ void __launch_bounds__(kThreads)
fwd_out_kernel(GdnProblem p, ExactWs ws, TIn* __restrict__ o) {
  __shared__ OutSmem sm;
  const int ci = blockIdx.x, h = blockIdx.y;
  if (ci >= *ws.ct.n_chunks) return;
  const int t0 = ws.ct.tok0[ci], L = ws.ct.len[ci];
  const int64_t ch = int64_t(ci) * p.Hv + h;
  if (threadIdx.x < 64) sm.cum[threadIdx.x] = ws.stats[ch * 256 + threadIdx.x];
  Frag<64, 128> a, b;
  a.zero(); b.zero();
  block_mm<64, 128>(a, ws.qn + ch * 8192, 128, 1, 64, ws.hs + ch * 16384, 128, 1, 128, 128, sm.sA, sm.sB);
  block_mm<64, 128>(b, ws.aqk + ch * 4096, 64, 1, 64, ws.vp + ch * 8192, 128, 1, 64, 64, sm.sA, sm.sB);
  const int w = warp_id(), l = lane_id();
#pragma unroll
  for (int ii = 0; ii < 8; ++ii) {
    const int i = w + 8 * ii;
    if (i >= L) continue;
    const float e = expf(sm.cum[i]);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj)
      stf(o + (int64_t(t0 + i) * p.Hv + h) * 128 + l + 32 * jj, e * a.v[ii][jj] + b.v[ii][jj]);
  }
}

// ------------------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------------------
struct BStateSmem {
  float ds[128 * 33];
  float dos[64 * 33];
  float doe[64 * 33];
  float dvs[64 * 33];
  float sA[128 * 17];
  float sB[16 * 33];
  float cum[64];
};

template <typename TIn>
__global__ void __launch_bounds__(kThreads)
bwd_state_kernel(GdnProblem p, ExactWs ws, const TIn* __restrict__ d_o, const float* __restrict__ dhT,
                 float* __restrict__ dh0) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  BStateSmem& sm = *reinterpret_cast<BStateSmem*>(smem_raw);
  const int h = blockIdx.x, s = blockIdx.y, j0 = blockIdx.z * 32;
  const int w = warp_id(), l = lane_id();
  const int64_t sbase = (int64_t(s) * p.Hv + h) * 16384;
  Frag<128, 32> dS;
#pragma unroll
  for (int ii = 0; ii < 16; ++ii) dS.v[ii][0] = dhT ? dhT[sbase + (w + 8 * ii) * 128 + j0 + l] : 0.f;
  const int c0 = ws.ct.seq_chunk0[s], c1 = ws.ct.seq_chunk0[s + 1];
  for (int ci = c1 - 1; ci >= c0; --ci) {
    const int64_t ch = int64_t(ci) * p.Hv + h;
    const int t0 = ws.ct.tok0[ci], L = ws.ct.len[ci];
    if (threadIdx.x < 64) sm.cum[threadIdx.x] = ws.stats[ch * 256 + threadIdx.x];
#pragma unroll
    for (int ii = 0; ii < 16; ++ii) {
      const int r = w + 8 * ii;
      ws.dh[ch * 16384 + r * 128 + j0 + l] = dS.v[ii][0];
      sm.ds[r * 33 + l] = dS.v[ii][0];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 64 * 32; idx += kThreads) {
      const int i = idx >> 5, j = idx & 31;
      const float x = i < L ? ldf(d_o + (int64_t(t0 + i) * p.Hv + h) * 128 + j0 + j) : 0.f;
      sm.dos[i * 33 + j] = x;
      sm.doe[i * 33 + j] = x * expf(sm.cum[i]);
    }
    __syncthreads();
    Frag<64, 32> a, b;
    a.zero(); b.zero();
    block_mm<64, 32>(a, ws.aqk + ch * 4096, 1, 64, 64, sm.dos, 33, 1, 64, 64, sm.sA, sm.sB);
    block_mm<64, 32>(b, ws.kn + ch * 8192, 128, 1, 64, sm.ds, 33, 1, 128, 128, sm.sA, sm.sB);
    const float cl = sm.cum[63];
#pragma unroll
    for (int ii = 0; ii < 8; ++ii) {
      const int c = w + 8 * ii;
      const float x = a.v[ii][0] + expf(cl - sm.cum[c]) * b.v[ii][0];
      ws.dvp[ch * 8192 + c * 128 + j0 + l] = x;
      sm.dvs[c * 33 + l] = x;
    }
    __syncthreads();
    Frag<128, 32> x1, x2;
    x1.zero(); x2.zero();
    block_mm<128, 32>(x1, ws.qn + ch * 8192, 1, 128, 128, sm.doe, 33, 1, 64, 64, sm.sA, sm.sB);
    block_mm<128, 32>(x2, ws.w + ch * 8192, 1, 128, 128, sm.dvs, 33, 1, 64, 64, sm.sA, sm.sB);
    const float gamma = expf(cl);
#pragma unroll
    for (int ii = 0; ii < 16; ++ii) dS.v[ii][0] = gamma * dS.v[ii][0] + x1.v[ii][0] - x2.v[ii][0];
    __syncthreads();
  }
  if (dh0) {
#pragma unroll
    for (int ii = 0; ii < 16; ++ii) dh0[sbase + (w + 8 * ii) * 128 + j0 + l] = dS.v[ii][0];
  }
}

template <typename TIn>
__global__ void __launch_bounds__(kThreads)
bwd_mm_kernel(GdnProblem p, ExactWs ws, const TIn* __restrict__ d_o) {
  __shared__ OutSmem sm;
  __shared__ float red[8];
  const int ci = blockIdx.x, h = blockIdx.y;
  if (ci >= *ws.ct.n_chunks) return;
  const int t0 = ws.ct.tok0[ci], L = ws.ct.len[ci];
  const int64_t ch = int64_t(ci) * p.Hv + h;
  const TIn* dO = d_o + (int64_t(t0) * p.Hv + h) * 128;
  const int64_t rs = int64_t(p.Hv) * 128;
  const int w = warp_id(), l = lane_id();
  Frag<64, 128> f;
  auto store = [&](float* dst, float sign) {
#pragma unroll
    for (int ii = 0; ii < 8; ++ii)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) dst[(w + 8 * ii) * 128 + l + 32 * jj] = sign * f.v[ii][jj];
  };
  f.zero();
  block_mm<64, 128>(f, dO, rs, 1, L, ws.hs + ch * 16384, 1, 128, 128, 128, sm.sA, sm.sB);
  store(ws.dqt + ch * 8192, 1.f);
  f.zero();
  block_mm<64, 128>(f, ws.dvp + ch * 8192, 128, 1, 64, ws.hs + ch * 16384, 1, 128, 128, 128, sm.sA, sm.sB);
  store(ws.dw + ch * 8192, -1.f);
  f.zero();
  block_mm<64, 128>(f, ws.vp + ch * 8192, 128, 1, 64, ws.dh + ch * 16384, 1, 128, 128, 128, sm.sA, sm.sB);
  store(ws.dkt + ch * 8192, 1.f);
  Frag<64, 64> a;
  a.zero();
  block_mm<64, 64>(a, dO, rs, 1, L, ws.vp + ch * 8192, 1, 128, 128, 128, sm.sA, sm.sB);
#pragma unroll
  for (int ii = 0; ii < 8; ++ii)
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int i = w + 8 * ii, j = l + 32 * jj;
      ws.daqk[ch * 4096 + i * 64 + j] = j <= i ? a.v[ii][jj] : 0.f;
    }
  float part = 0.f;
  for (int idx = threadIdx.x; idx < 16384; idx += kThreads)
    part = fmaf(ws.hs[ch * 16384 + idx], ws.dh[ch * 16384 + idx], part);
  part = block_sum(part, red);
  if (threadIdx.x == 0) ws.dgam[ch] = part;
}

struct IntraSmem {
  float qn[64 * 129];
  float kn[64 * 129];
  float vv[64 * 129];   // v, later beta * k
  float tm[64 * 65];    // T, later R
  float x[64 * 65];     // dT, later P = dL * Gamma
  float y[64 * 65];     // T^T dT, later Qm = dA_qk * Gamma
  float sA[64 * 17];
  float sB[16 * 129];
  float cum[64], ecum[64], edec[64], beta[64], rq[64], rk[64];
  float dbeta[64], dcum[64];
  float red[8];
};

template <typename TIn>
__global__ void __launch_bounds__(kThreads)
bwd_intra_kernel(GdnProblem p, ExactWs ws, TIn* __restrict__ dq, TIn* __restrict__ dk,
                 TIn* __restrict__ dv, float* __restrict__ dg, TIn* __restrict__ dbeta) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  IntraSmem& sm = *reinterpret_cast<IntraSmem*>(smem_raw);
  const int ci = blockIdx.x, h = blockIdx.y;
  if (ci >= *ws.ct.n_chunks) return;
  const int t0 = ws.ct.tok0[ci], L = ws.ct.len[ci], hk = h / p.group;
  const int64_t ch = int64_t(ci) * p.Hv + h;
  const int w = warp_id(), l = lane_id();
  const TIn* v = static_cast<const TIn*>(p.v) + (int64_t(t0) * p.Hv + h) * 128;
  const int64_t vrs = int64_t(p.Hv) * 128;

  for (int idx = threadIdx.x; idx < 64 * 128; idx += kThreads) {
    const int i = idx >> 7, c = idx & 127;
    sm.qn[i * 129 + c] = ws.qn[ch * 8192 + idx];
    sm.kn[i * 129 + c] = ws.kn[ch * 8192 + idx];
    sm.vv[i * 129 + c] = i < L ? ldf(v + i * vrs + c) : 0.f;
  }
  for (int idx = threadIdx.x; idx < 64 * 64; idx += kThreads) sm.tm[(idx >> 6) * 65 + (idx & 63)] = ws.tinv[ch * 4096 + idx];
  if (threadIdx.x < 64) {
    const int i = threadIdx.x;
    const float* st = ws.stats + ch * 256;
    sm.cum[i] = st[i]; sm.rq[i] = st[64 + i]; sm.rk[i] = st[128 + i]; sm.beta[i] = st[192 + i];
    sm.ecum[i] = expf(st[i]);
    sm.edec[i] = expf(st[63] - st[i]);
  }
  __syncthreads();

  Frag<64, 128> dqn, dkn;
  dqn.zero(); dkn.zero();
  float dbeta_r[8], dcum_r[8];
#pragma unroll
  for (int ii = 0; ii < 8; ++ii) { dbeta_r[ii] = 0.f; dcum_r[ii] = 0.f; }

  // (1) dBv = T^T dU -> dv, dbeta; dBk = T^T dW -> dk, dbeta, dcum
  {
    Frag<64, 128> f;
    f.zero();
    block_mm<64, 128>(f, sm.tm, 1, 65, 64, ws.dvp + ch * 8192, 128, 1, 64, 64, sm.sA, sm.sB);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii) {
      const int i = w + 8 * ii;
      float part = 0.f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int c = l + 32 * jj;
        part = fmaf(f.v[ii][jj], sm.vv[i * 129 + c], part);
        if (i < L) stf(dv + (int64_t(t0 + i) * p.Hv + h) * 128 + c, sm.beta[i] * f.v[ii][jj]);
      }
      dbeta_r[ii] += warp_sum(part);
    }
    f.zero();
    block_mm<64, 128>(f, sm.tm, 1, 65, 64, ws.dw + ch * 8192, 128, 1, 64, 64, sm.sA, sm.sB);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii) {
      const int i = w + 8 * ii;
      const float be = sm.beta[i] * sm.ecum[i];
      float part = 0.f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int c = l + 32 * jj;
        part = fmaf(f.v[ii][jj], sm.kn[i * 129 + c], part);
        dkn.v[ii][jj] += be * f.v[ii][jj];
      }
      part = warp_sum(part);
      dbeta_r[ii] += sm.ecum[i] * part;
      dcum_r[ii] += be * part;
    }
  }
  // dT = dU (beta V)^T + dW (beta e^cum K)^T, lower triangle incl. diagonal
  {
    Frag<64, 64> a, b;
    a.zero(); b.zero();
    block_mm<64, 64>(a, ws.dvp + ch * 8192, 128, 1, 64, sm.vv, 1, 129, 128, 128, sm.sA, sm.sB);
    block_mm<64, 64>(b, ws.dw + ch * 8192, 128, 1, 64, sm.kn, 1, 129, 128, 128, sm.sA, sm.sB);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int i = w + 8 * ii, j = l + 32 * jj;
        sm.x[i * 65 + j] = j <= i ? sm.beta[j] * (a.v[ii][jj] + sm.ecum[j] * b.v[ii][jj]) : 0.f;
      }
  }
  __syncthreads();
  // (2) dL = -(T^T dT T^T), strictly lower
  Frag<64, 64> dL;
  {
    Frag<64, 64> y;
    y.zero();
    block_mm<64, 64>(y, sm.tm, 1, 65, 64, sm.x, 65, 1, 64, 64, sm.sA, sm.sB);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) sm.y[(w + 8 * ii) * 65 + l + 32 * jj] = y.v[ii][jj];
    __syncthreads();
    dL.zero();
    block_mm<64, 64>(dL, sm.y, 65, 1, 64, sm.tm, 1, 65, 64, 64, sm.sA, sm.sB);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii)
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int i = w + 8 * ii, j = l + 32 * jj;
        dL.v[ii][jj] = j < i ? -dL.v[ii][jj] : 0.f;
      }
  }
  // (3) through L = beta (k k^T) Gamma and A_qk = (q k^T) Gamma
  {
    Frag<64, 64> kk, qk;
    kk.zero(); qk.zero();
    block_mm<64, 64>(kk, sm.kn, 129, 1, 64, sm.kn, 1, 129, 128, 128, sm.sA, sm.sB);
    block_mm<64, 64>(qk, sm.qn, 129, 1, 64, sm.kn, 1, 129, 128, 128, sm.sA, sm.sB);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii) {
      const int i = w + 8 * ii;
      float part = 0.f;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int j = l + 32 * jj;
        const float gam = j <= i ? expf(sm.cum[i] - sm.cum[j]) : 0.f;
        const float P = dL.v[ii][jj] * gam;
        const float daqk = ws.daqk[ch * 4096 + i * 64 + j];
        part = fmaf(P, kk.v[ii][jj], part);
        sm.x[i * 65 + j] = P;
        sm.y[i * 65 + j] = daqk * gam;
        sm.tm[i * 65 + j] = P * sm.beta[i] * kk.v[ii][jj] + daqk * qk.v[ii][jj] * gam;  // R
      }
      dbeta_r[ii] += warp_sum(part);
    }
  }
  for (int idx = threadIdx.x; idx < 64 * 128; idx += kThreads) {
    const int i = idx >> 7, c = idx & 127;
    sm.vv[i * 129 + c] = sm.beta[i] * sm.kn[i * 129 + c];
  }
  __syncthreads();
  // (4) dk += diag(beta) P K + P^T (beta K);  dq += Qm K;  dk += Qm^T Q
  {
    Frag<64, 128> f;
    f.zero();
    block_mm<64, 128>(f, sm.x, 65, 1, 64, sm.kn, 129, 1, 64, 64, sm.sA, sm.sB);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) dkn.v[ii][jj] += sm.beta[w + 8 * ii] * f.v[ii][jj];
    block_mm<64, 128>(dkn, sm.x, 1, 65, 64, sm.vv, 129, 1, 64, 64, sm.sA, sm.sB);
    block_mm<64, 128>(dqn, sm.y, 65, 1, 64, sm.kn, 129, 1, 64, 64, sm.sA, sm.sB);
    block_mm<64, 128>(dkn, sm.y, 1, 65, 64, sm.qn, 129, 1, 64, 64, sm.sA, sm.sB);
  }
  if (threadIdx.x < 64) {  // dcum_i += sum_j R_ij - sum_j R_ji
    const int i = threadIdx.x;
    float a = 0.f;
    for (int j = 0; j < 64; ++j) a += sm.tm[i * 65 + j] - sm.tm[j * 65 + i];
    sm.dcum[i] = a;
  }
  __syncthreads();
  // (5) q~ = e^cum q, k~ = e^(cl - cum) k, gamma = e^cl
  float dcl_part = 0.f;
#pragma unroll
  for (int ii = 0; ii < 8; ++ii) {
    const int i = w + 8 * ii;
    float pq = 0.f, pk = 0.f;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int c = l + 32 * jj;
      const float dqt = ws.dqt[ch * 8192 + i * 128 + c];
      const float dkt = ws.dkt[ch * 8192 + i * 128 + c];
      dqn.v[ii][jj] += sm.ecum[i] * dqt;
      dkn.v[ii][jj] += sm.edec[i] * dkt;
      pq = fmaf(dqt, sm.qn[i * 129 + c], pq);
      pk = fmaf(dkt, sm.kn[i * 129 + c], pk);
    }
    pq = warp_sum(pq) * sm.ecum[i];
    pk = warp_sum(pk) * sm.edec[i];
    dcum_r[ii] += pq - pk;
    dcl_part += pk;
  }
  if (l == 0) {
#pragma unroll
    for (int ii = 0; ii < 8; ++ii) {
      const int i = w + 8 * ii;
      sm.dcum[i] += dcum_r[ii];
      sm.dbeta[i] = dbeta_r[ii];
    }
  }
  // every lane of a warp holds the same dcl_part
  if (l == 0) sm.red[w] = dcl_part;
  __syncthreads();
  if (threadIdx.x == 0) {
    float dcl = 0.f;
    for (int i = 0; i < 8; ++i) dcl += sm.red[i];
    dcl += ws.dgam[ch] * expf(sm.cum[63]);
    sm.dcum[63] += dcl;
    double acc = 0.0;  // dg_t = sum_{i >= t} dcum_i
    for (int i = 63; i >= 0; --i) {
      acc += double(sm.dcum[i]);
      if (i < L) dg[int64_t(t0 + i) * p.Hv + h] = float(acc);
    }
  }
  if (threadIdx.x < 64 && threadIdx.x < L) stf(dbeta + int64_t(t0 + threadIdx.x) * p.Hv + h, sm.dbeta[threadIdx.x]);
  // (6) l2norm backward: dx = r dy - x r^3 (x . dy)
  const TIn* q = static_cast<const TIn*>(p.q) + (int64_t(t0) * p.Hk + hk) * 128;
  const TIn* k = static_cast<const TIn*>(p.k) + (int64_t(t0) * p.Hk + hk) * 128;
  const int64_t krs = int64_t(p.Hk) * 128;
#pragma unroll
  for (int ii = 0; ii < 8; ++ii) {
    const int i = w + 8 * ii;
    if (i >= L) continue;
    float xq[4], xk[4], pq = 0.f, pk = 0.f;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int c = l + 32 * jj;
      xq[jj] = ldf(q + i * krs + c);
      xk[jj] = ldf(k + i * krs + c);
      dqn.v[ii][jj] *= p.scale;
      pq = fmaf(xq[jj], dqn.v[ii][jj], pq);
      pk = fmaf(xk[jj], dkn.v[ii][jj], pk);
    }
    pq = warp_sum(pq);
    pk = warp_sum(pk);
    const float rq = sm.rq[i], rk = sm.rk[i];
    const float rq3 = rq * rq * rq, rk3 = rk * rk * rk;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int c = l + 32 * jj;
      const float gq = rq * dqn.v[ii][jj] - xq[jj] * rq3 * pq;
      const float gk = rk * dkn.v[ii][jj] - xk[jj] * rk3 * pk;
      if (p.group == 1) {
        stf(dq + (int64_t(t0 + i) * p.Hk + hk) * 128 + c, gq);
        stf(dk + (int64_t(t0 + i) * p.Hk + hk) * 128 + c, gk);
      } else {
        ws.dqh[(int64_t(t0 + i) * p.Hv + h) * 128 + c] = gq;
        ws.dkh[(int64_t(t0 + i) * p.Hv + h) * 128 + c] = gk;
      }
    }
  }
}

template <typename TIn>
__global__ void __launch_bounds__(kThreads)
bwd_gqa_kernel(GdnProblem p, ExactWs ws, TIn* __restrict__ dq, TIn* __restrict__ dk) {
  const int64_t n = p.tokens * p.Hk * 128;
  for (int64_t idx = int64_t(blockIdx.x) * kThreads + threadIdx.x; idx < n; idx += int64_t(gridDim.x) * kThreads) {
    const int64_t c = idx & 127, th = idx >> 7, hk = th % p.Hk, tok = th / p.Hk;
    float aq = 0.f, ak = 0.f;
    for (int r = 0; r < p.group; ++r) {
      const int64_t src = (tok * p.Hv + hk * p.group + r) * 128 + c;
      aq += ws.dqh[src];
      ak += ws.dkh[src];
    }
    stf(dq + idx, aq);
    stf(dk + idx, ak);
  }
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    return RB2_ECUDA;
  }
  return RB2_OK;
}

}  // namespace

int launch_chunk_table(const GdnProblem& p, const ChunkTable& ct, cudaStream_t s) {
  { ProfScope ps_("gdn_chunk_table", s); chunk_table_kernel<<<1, 1024, 0, s>>>(p.cu_seqlens, p.n_seqs, p.T, p.max_chunks, ct); }
  RB2_CHECK_LAUNCH("gdn chunk table");
  return RB2_OK;
}

template <typename TIn>
int exact_forward(const GdnProblem& p, ExactWs& ws, TIn* o, float* hT, cudaStream_t s) {
  int rc = launch_chunk_table(p, ws.ct, s);
  if (rc) return rc;
  RB2_CUDA(cudaMemsetAsync(ws.err, 0, sizeof(int), s), "gdn exact: clear status");  // no bounded waits here
  if (p.max_chunks > 0) {
    if ((rc = set_smem(fwd_prep_kernel<TIn>, sizeof(PrepSmem)))) return rc;
    ProfScope ps_("gdn_exact_fwd_prep", s);
    fwd_prep_kernel<TIn><<<dim3(p.max_chunks, p.Hv), kThreads, sizeof(PrepSmem), s>>>(p, ws);
    RB2_CHECK_LAUNCH("gdn exact fwd_prep");
  }
  if ((rc = set_smem(fwd_state_kernel, sizeof(StateSmem)))) return rc;
  { ProfScope ps_("gdn_exact_fwd_state", s); fwd_state_kernel<<<dim3(p.Hv, unsigned(p.n_seqs), 4), kThreads, sizeof(StateSmem), s>>>(p, ws, hT); }
  RB2_CHECK_LAUNCH("gdn exact fwd_state");
  if (p.max_chunks > 0) {
    ProfScope ps_("gdn_exact_fwd_out", s);
    fwd_out_kernel<TIn><<<dim3(p.max_chunks, p.Hv), kThreads, 0, s>>>(p, ws, o);
    RB2_CHECK_LAUNCH("gdn exact fwd_out");
  }
  return RB2_OK;
}

template <typename TIn>
int exact_backward(const GdnProblem& p, ExactWs& ws, const TIn* d_o, const float* dhT, TIn* dq, TIn* dk,
                   TIn* dv, float* dg, TIn* dbeta, float* dh0, cudaStream_t s) {
  int rc;
  if ((rc = set_smem(bwd_state_kernel<TIn>, sizeof(BStateSmem)))) return rc;
  { ProfScope ps_("gdn_exact_bwd_state", s); bwd_state_kernel<TIn><<<dim3(p.Hv, unsigned(p.n_seqs), 4), kThreads, sizeof(BStateSmem), s>>>(p, ws, d_o, dhT, dh0); }
  RB2_CHECK_LAUNCH("gdn exact bwd_state");
  if (p.max_chunks > 0) {
    { ProfScope ps_("gdn_exact_bwd_mm", s); bwd_mm_kernel<TIn><<<dim3(p.max_chunks, p.Hv), kThreads, 0, s>>>(p, ws, d_o); }
    RB2_CHECK_LAUNCH("gdn exact bwd_mm");
    if ((rc = set_smem(bwd_intra_kernel<TIn>, sizeof(IntraSmem)))) return rc;
    { ProfScope ps_("gdn_exact_bwd_intra", s); bwd_intra_kernel<TIn><<<dim3(p.max_chunks, p.Hv), kThreads, sizeof(IntraSmem), s>>>(p, ws, dq, dk, dv, dg, dbeta); }
    RB2_CHECK_LAUNCH("gdn exact bwd_intra");
    if (p.group > 1) {
      { ProfScope ps_("gdn_exact_bwd_gqa", s); bwd_gqa_kernel<TIn><<<148 * 8, kThreads, 0, s>>>(p, ws, dq, dk); }
      RB2_CHECK_LAUNCH("gdn exact bwd_gqa");
    }
  }
  return RB2_OK;
}

template int exact_forward<float>(const GdnProblem&, ExactWs&, float*, float*, cudaStream_t);
template int exact_forward<__nv_bfloat16>(const GdnProblem&, ExactWs&, __nv_bfloat16*, float*, cudaStream_t);
template int exact_backward<float>(const GdnProblem&, ExactWs&, const float*, const float*, float*, float*,
                                   float*, float*, float*, float*, cudaStream_t);
template int exact_backward<__nv_bfloat16>(const GdnProblem&, ExactWs&, const __nv_bfloat16*, const float*,
                                           __nv_bfloat16*, __nv_bfloat16*, __nv_bfloat16*, float*,
                                           __nv_bfloat16*, float*, cudaStream_t);

}  // namespace rb2
