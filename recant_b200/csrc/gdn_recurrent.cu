// Token-by-token gated delta rule with a carried state: the decode / short-chunk step of the serving
// loop (recant/serve/engine.py:107-119 -> GatedDeltaNet.forward with a LayerCache, layers.py:148-182
// -> gdn_core(..., initial_state=cache.rec_state, output_final_state=True), ops.py:21-54 and 62-67).
//
// gdn_torch pads a short call to one 64-token chunk; for one chunk its algebra reduces to the plain
// recurrence, which is what this kernel runs, in fp32:
//   q^ = q rsqrt(sum q^2 + 1e-6) dk^-1/2,  k^ = k rsqrt(sum k^2 + 1e-6)            (ops.py:18-19, 26-27)
//   S <- e^{g_t} S;  v'_t = beta_t (v_t - S^T k^_t);  S <- S + k^_t v'_t^T;  o_t = S^T q^_t
// State layout [seq, Hv, dk, dv] fp32 as the reference's cache (layers.py:111-130). The columns of S
// evolve independently, so one CTA owns 32 of them for one (sequence, value head): 128 threads, a
// thread holds 32 rows of one column in registers; two cross-warp sums per token (S^T k, S^T q).
// The state is read once and written once per call; the final state may overwrite the initial one.
#include "common.cuh"

namespace rb2 {
namespace {

constexpr int kD = 128, kCols = 32, kThr = 128;

__device__ __forceinline__ float ldf(const float* p) { return *p; }
__device__ __forceinline__ float ldf(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void stf(float* p, float v) { *p = v; }
__device__ __forceinline__ void stf(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kThr) gdn_recurrent_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                             const T* __restrict__ v, const float* __restrict__ g,
                                                             const T* __restrict__ beta, const float* h0,
                                                             const int64_t* __restrict__ cu, int Tn, int Hk, int Hv,
                                                             float scale, T* __restrict__ o, float* hT) {
  const int cb = blockIdx.x % (kD / kCols);
  const int sh = blockIdx.x / (kD / kCols);  // sequence x value head
  const int n = sh / Hv, h = sh % Hv, hk = h / (Hv / Hk);
  const int tid = threadIdx.x, j = tid & 31, rq = tid >> 5;
  const int col = cb * kCols + j;
  __shared__ float kn[kD], qn[kD], part[2][4], red[2][4][kCols];
  const int64_t t0 = cu ? cu[n] : int64_t(n) * Tn, t1 = cu ? cu[n + 1] : t0 + Tn;
  const size_t sbase = (size_t(n) * Hv + h) * kD * kD + col;
  float S[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) S[i] = h0 ? h0[sbase + size_t(rq * 32 + i) * kD] : 0.f;
  for (int64_t t = t0; t < t1; ++t) {
    const float kv = ldf(k + (t * Hk + hk) * kD + tid), qv = ldf(q + (t * Hk + hk) * kD + tid);
    const float sk = warp_sum(kv * kv), sq = warp_sum(qv * qv);
    if (j == 0) {
      part[0][rq] = sk;
      part[1][rq] = sq;
    }
    __syncthreads();
    kn[tid] = kv * rsqrtf(part[0][0] + part[0][1] + part[0][2] + part[0][3] + 1e-6f);
    qn[tid] = qv * rsqrtf(part[1][0] + part[1][1] + part[1][2] + part[1][3] + 1e-6f) * scale;
    __syncthreads();
    const float dec = expf(g[t * Hv + h]), bt = ldf(beta + t * Hv + h);
    const float vj = ldf(v + (t * Hv + h) * kD + col);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      S[i] *= dec;
      dot = fmaf(S[i], kn[rq * 32 + i], dot);
    }
    red[0][rq][j] = dot;
    __syncthreads();
    const float vp = bt * (vj - (red[0][0][j] + red[0][1][j] + red[0][2][j] + red[0][3][j]));
    float oj = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      S[i] = fmaf(kn[rq * 32 + i], vp, S[i]);
      oj = fmaf(S[i], qn[rq * 32 + i], oj);
    }
    red[1][rq][j] = oj;
    __syncthreads();
    if (rq == 0) stf(o + (t * Hv + h) * kD + col, red[1][0][j] + red[1][1][j] + red[1][2][j] + red[1][3][j]);
  }
  if (hT) {
#pragma unroll
    for (int i = 0; i < 32; ++i) hT[sbase + size_t(rq * 32 + i) * kD] = S[i];
  }
}

}  // namespace
}  // namespace rb2

using namespace rb2;

extern "C" int rb2_gdn_recurrent_fwd(const void* q, const void* k, const void* v, const float* g, const void* beta,
                                     const float* h0, const int64_t* cu_seqlens, int B, int T, int n_seqs, int Hk,
                                     int Hv, int dk, int dv, int dtype, float scale, void* o, float* hT,
                                     void* stream) {
  RB2_CHECK_ARG(dk == kD && dv == kD, "gdn_recurrent: head dims must be 128 (dk=%d dv=%d)", dk, dv);
  RB2_CHECK_ARG(B >= 1 && T >= 0 && Hk >= 1 && Hv >= Hk && Hv % Hk == 0, "gdn_recurrent: bad sizes B=%d T=%d Hk=%d Hv=%d",
                B, T, Hk, Hv);
  RB2_CHECK_ARG(dtype == RB2_F32 || dtype == RB2_BF16, "gdn_recurrent: dtype");
  RB2_CHECK_ARG(cu_seqlens == nullptr ? n_seqs == B : (B == 1 && n_seqs >= 1),
                "gdn_recurrent: cu_seqlens needs B == 1; without it n_seqs == B");
  RB2_CHECK_ARG(q && k && v && g && beta && o, "gdn_recurrent: null pointer");
  const int64_t ctas = int64_t(n_seqs) * Hv * (kD / kCols);
  RB2_CHECK_ARG(ctas < (int64_t(1) << 31), "gdn_recurrent: too many sequences x heads");
  if (T == 0 && hT == nullptr) return RB2_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ProfScope ps_("gdn_recurrent", s);
  if (dtype == RB2_BF16) {
    using T16 = __nv_bfloat16;
    gdn_recurrent_kernel<T16><<<unsigned(ctas), kThr, 0, s>>>(
        static_cast<const T16*>(q), static_cast<const T16*>(k), static_cast<const T16*>(v), g,
        static_cast<const T16*>(beta), h0, cu_seqlens, T, Hk, Hv, scale, static_cast<T16*>(o), hT);
  } else {
    gdn_recurrent_kernel<float><<<unsigned(ctas), kThr, 0, s>>>(
        static_cast<const float*>(q), static_cast<const float*>(k), static_cast<const float*>(v), g,
        static_cast<const float*>(beta), h0, cu_seqlens, T, Hk, Hv, scale, static_cast<float*>(o), hT);
  }
  RB2_CHECK_LAUNCH("gdn_recurrent");
  return RB2_OK;
}
