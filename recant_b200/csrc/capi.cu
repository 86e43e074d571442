// extern "C" entry points of the GDN op: argument checks, workspace carving, path dispatch.
#include <cstdarg>
#include <cstdio>

#include "gdn_common.cuh"

namespace rb2 {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

template <typename TIn>
int exact_forward(const GdnProblem& p, ExactWs& ws, TIn* o, float* hT, cudaStream_t s);
template <typename TIn>
int exact_backward(const GdnProblem& p, ExactWs& ws, const TIn* d_o, const float* dhT, TIn* dq, TIn* dk,
                   TIn* dv, float* dg, TIn* dbeta, float* dh0, cudaStream_t s);

int fast_forward(const GdnProblem& p, void* ws, void* o, float* hT, cudaStream_t s);
int fast_backward(const GdnProblem& p, void* ws, void* scratch, const void* d_o, const float* dhT, void* dq, void* dk,
                  void* dv, float* dg, void* dbeta, float* dh0, cudaStream_t s);
void fast_workspace_split(int64_t tokens, int64_t n_seqs, int Hk, int Hv, int max_chunks, size_t* saved,
                          size_t* scratch);

namespace {

int resolve_path(int dtype, int path) {
  if (path == RB2_GDN_AUTO) return dtype == RB2_BF16 ? RB2_GDN_FAST : RB2_GDN_EXACT;
  return path;
}

int check_problem(int64_t B, int64_t T, int64_t n_seqs, int Hk, int Hv, int dk, int dv, int dtype,
                  int path, bool varlen) {
  RB2_CHECK_ARG(dtype == RB2_F32 || dtype == RB2_BF16, "gdn: dtype must be RB2_F32 or RB2_BF16");
  RB2_CHECK_ARG(B >= 1 && T >= 0 && n_seqs >= 1, "gdn: bad sizes B=%lld T=%lld N=%lld", (long long)B,
                (long long)T, (long long)n_seqs);
  RB2_CHECK_ARG(Hk >= 1 && Hv >= 1 && Hv % Hk == 0, "gdn: Hv (%d) must be a multiple of Hk (%d)", Hv, Hk);
  RB2_CHECK_ARG(varlen ? B == 1 : n_seqs == B, "gdn: cu_seqlens needs B == 1; otherwise n_seqs == B");
  RB2_CHECK_ARG(n_seqs <= 65535 && Hv <= 65535, "gdn: too many sequences/heads");
  RB2_CHECK_ARG(path == RB2_GDN_AUTO || path == RB2_GDN_EXACT || path == RB2_GDN_FAST, "gdn: bad path %d", path);
  if (dk != 128 || dv != 128) {
    set_error("gdn: head dims dk=%d dv=%d unsupported (need 128)", dk, dv);
    return RB2_EUNSUPPORTED;
  }
  if (resolve_path(dtype, path) == RB2_GDN_FAST && dtype != RB2_BF16) {
    set_error("gdn: the tensor-core path needs bf16 inputs");
    return RB2_EINVAL;
  }
  return RB2_OK;
}

GdnProblem make_problem(const void* q, const void* k, const void* v, const float* g, const void* beta,
                        const float* h0, const int64_t* cu, int64_t B, int64_t T, int64_t n_seqs, int Hk,
                        int Hv, int dtype, int path, float scale) {
  GdnProblem p;
  p.q = q; p.k = k; p.v = v; p.g = g; p.beta = beta; p.h0 = h0; p.cu_seqlens = cu;
  p.B = B; p.T = T; p.n_seqs = n_seqs; p.tokens = B * T;
  p.Hk = Hk; p.Hv = Hv; p.group = Hv / Hk;
  p.dtype = dtype; p.path = resolve_path(dtype, path); p.scale = scale;
  p.max_chunks = gdn_max_chunks(p.tokens, n_seqs);
  return p;
}

// The tensor-core path moves rows of q, k, v, dO, o with 16-byte (bulk) copies and writes dq, dk,
// dv in 4-byte pairs.
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

size_t exact_ws_bytes(const GdnProblem& p, ExactWs* out, void* base) {
  Carver c(base);
  ExactWs w;
  size_t n = carve_exact(c, w, p.tokens, p.n_seqs, p.Hv, p.max_chunks, p.group > 1);
  if (out) *out = w;
  return n;
}

}  // namespace
}  // namespace rb2

using namespace rb2;

extern "C" const char* rb2_last_error(void) { return g_err; }

extern "C" int rb2_status_read(const void* status_word, int* code, int clear, void* stream) {
  RB2_CHECK_ARG(status_word && code && (reinterpret_cast<uintptr_t>(status_word) & 3) == 0,
                "status_read: null or misaligned pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  RB2_CUDA(cudaStreamSynchronize(s), "status_read: synchronize");
  RB2_CUDA(cudaMemcpy(code, status_word, sizeof(int), cudaMemcpyDeviceToHost), "status_read: copy");
  if (clear) RB2_CUDA(cudaMemset(const_cast<void*>(status_word), 0, sizeof(int)), "status_read: clear");
  return RB2_OK;
}
extern "C" const char* rb2_version(void) { return "recant_b200 0.1 (sm_100a)"; }

namespace rb2 {
namespace {
// Bytes of the workspace part the forward fills and the backward reads ("saved") and of the part
// only the backward uses ("scratch"); the single-buffer layout is saved followed by scratch.
void ws_split(const GdnProblem& p, size_t* saved, size_t* scratch) {
  if (p.path == RB2_GDN_FAST) {
    fast_workspace_split(p.tokens, p.n_seqs, p.Hk, p.Hv, p.max_chunks, saved, scratch);
  } else {
    *saved = exact_ws_bytes(p, nullptr, nullptr);
    *scratch = 0;
  }
}
}  // namespace
}  // namespace rb2

extern "C" size_t rb2_gdn_workspace_size(int64_t B, int64_t T, int64_t n_seqs, int Hk, int Hv, int dk, int dv,
                                         int dtype, int path) {
  if (check_problem(B, T, n_seqs, Hk, Hv, dk, dv, dtype, path, n_seqs != B || B == 1)) return 0;
  GdnProblem p = make_problem(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, B, T, n_seqs, Hk,
                              Hv, dtype, path, 1.f);
  size_t saved, scratch;
  ws_split(p, &saved, &scratch);
  return saved + scratch;
}

extern "C" int rb2_gdn_workspace_split(int64_t B, int64_t T, int64_t n_seqs, int Hk, int Hv, int dk, int dv,
                                       int dtype, int path, size_t* saved_bytes, size_t* scratch_bytes) {
  int rc = check_problem(B, T, n_seqs, Hk, Hv, dk, dv, dtype, path, n_seqs != B || B == 1);
  if (rc) return rc;
  RB2_CHECK_ARG(saved_bytes && scratch_bytes, "gdn_workspace_split: null output pointer");
  GdnProblem p = make_problem(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, B, T, n_seqs, Hk,
                              Hv, dtype, path, 1.f);
  ws_split(p, saved_bytes, scratch_bytes);
  return RB2_OK;
}

namespace rb2 {
namespace {
int gdn_fwd_impl(const void* q, const void* k, const void* v, const float* g, const void* beta, const float* h0,
                 const int64_t* cu_seqlens, int64_t B, int64_t T, int64_t n_seqs, int Hk, int Hv, int dk, int dv,
                 int dtype, int path, float scale, void* o, float* hT, void* ws, size_t ws_bytes, void* stream,
                 int stages, int walk) {
  int rc = check_problem(B, T, n_seqs, Hk, Hv, dk, dv, dtype, path, cu_seqlens != nullptr);
  if (rc) return rc;
  RB2_CHECK_ARG(ws != nullptr, "gdn_fwd: null workspace");
  RB2_CHECK_ARG(stages >= 1 && stages <= 3 && walk >= 0 && walk <= 2, "gdn_fwd: bad stages/walk");
  RB2_CHECK_ARG(B * T == 0 || (q && k && v && g && beta && (o || walk != 0 || !(stages & 2))),
                "gdn_fwd: null input/output pointer");
  GdnProblem p = make_problem(q, k, v, g, beta, h0, cu_seqlens, B, T, n_seqs, Hk, Hv, dtype, path, scale);
  p.stages = stages;
  p.walk = walk;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  size_t saved, scratch;
  ws_split(p, &saved, &scratch);
  if (p.path == RB2_GDN_FAST) {
    RB2_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o) && aligned16(ws),
                  "gdn_fwd: q, k, v, o and ws must be 16-byte aligned on the tensor-core path");
    if (ws_bytes < saved) {
      set_error("gdn_fwd: workspace too small");
      return RB2_EWORKSPACE;
    }
    return fast_forward(p, ws, o, hT, s);
  }
  if (stages != 3 || walk != 0) {
    set_error("gdn_fwd: stage/walk selection needs the tensor-core path");
    return RB2_EUNSUPPORTED;
  }
  ExactWs w;
  if (ws_bytes < exact_ws_bytes(p, &w, ws)) {
    set_error("gdn_fwd: workspace too small");
    return RB2_EWORKSPACE;
  }
  if (dtype == RB2_BF16) return exact_forward<__nv_bfloat16>(p, w, static_cast<__nv_bfloat16*>(o), hT, s);
  return exact_forward<float>(p, w, static_cast<float*>(o), hT, s);
}

int gdn_bwd_impl(const void* q, const void* k, const void* v, const float* g, const void* beta, const float* h0,
                 const int64_t* cu_seqlens, int64_t B, int64_t T, int64_t n_seqs, int Hk, int Hv, int dk, int dv,
                 int dtype, int path, float scale, const void* d_o, const float* dhT, void* dq, void* dk_out,
                 void* dv_out, float* dg, void* dbeta, float* dh0, void* ws, size_t ws_bytes, void* scratch,
                 size_t scratch_bytes, void* stream, int stages, int walk) {
  int rc = check_problem(B, T, n_seqs, Hk, Hv, dk, dv, dtype, path, cu_seqlens != nullptr);
  if (rc) return rc;
  RB2_CHECK_ARG(ws != nullptr, "gdn_bwd: null workspace");
  RB2_CHECK_ARG(stages >= 1 && stages <= 3 && walk >= 0 && walk <= 1, "gdn_bwd: bad stages/walk");
  RB2_CHECK_ARG(B * T == 0 || d_o, "gdn_bwd: null dO");
  RB2_CHECK_ARG(B * T == 0 || !(stages & 2) || (dq && dk_out && dv_out && dg && dbeta), "gdn_bwd: null gradient pointer");
  GdnProblem p = make_problem(q, k, v, g, beta, h0, cu_seqlens, B, T, n_seqs, Hk, Hv, dtype, path, scale);
  p.stages = stages;
  p.walk = walk;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  size_t saved, need_scratch;
  ws_split(p, &saved, &need_scratch);
  if (p.path == RB2_GDN_FAST) {
    RB2_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(d_o) && aligned16(dq) &&
                      aligned16(dk_out) && aligned16(dv_out) && aligned16(ws) && aligned16(scratch),
                  "gdn_bwd: q, k, v, dO, dq, dk, dv, ws and scratch must be 16-byte aligned on the tensor-core path");
    if (scratch ? (ws_bytes < saved || scratch_bytes < need_scratch) : ws_bytes < saved + need_scratch) {
      set_error("gdn_bwd: workspace too small");
      return RB2_EWORKSPACE;
    }
    return fast_backward(p, ws, scratch, d_o, dhT, dq, dk_out, dv_out, dg, dbeta, dh0, s);
  }
  if (stages != 3 || walk != 0) {
    set_error("gdn_bwd: stage/walk selection needs the tensor-core path");
    return RB2_EUNSUPPORTED;
  }
  ExactWs w;
  if (ws_bytes < exact_ws_bytes(p, &w, ws)) {
    set_error("gdn_bwd: workspace too small");
    return RB2_EWORKSPACE;
  }
  if (dtype == RB2_BF16) {
    using T16 = __nv_bfloat16;
    return exact_backward<T16>(p, w, static_cast<const T16*>(d_o), dhT, static_cast<T16*>(dq),
                               static_cast<T16*>(dk_out), static_cast<T16*>(dv_out), dg, static_cast<T16*>(dbeta),
                               dh0, s);
  }
  return exact_backward<float>(p, w, static_cast<const float*>(d_o), dhT, static_cast<float*>(dq),
                               static_cast<float*>(dk_out), static_cast<float*>(dv_out), dg,
                               static_cast<float*>(dbeta), dh0, s);
}
}  // namespace
}  // namespace rb2

extern "C" int rb2_gdn_fwd(const void* q, const void* k, const void* v, const float* g, const void* beta,
                           const float* h0, const int64_t* cu_seqlens, int64_t B, int64_t T, int64_t n_seqs,
                           int Hk, int Hv, int dk, int dv, int dtype, int path, float scale, void* o,
                           float* hT, void* ws, size_t ws_bytes, void* stream) {
  return gdn_fwd_impl(q, k, v, g, beta, h0, cu_seqlens, B, T, n_seqs, Hk, Hv, dk, dv, dtype, path, scale, o, hT, ws,
                      ws_bytes, stream, 3, 0);
}

extern "C" int rb2_gdn_fwd_ex(const void* q, const void* k, const void* v, const float* g, const void* beta,
                              const float* h0, const int64_t* cu_seqlens, int64_t B, int64_t T, int64_t n_seqs,
                              int Hk, int Hv, int dk, int dv, int dtype, int path, float scale, void* o,
                              float* hT, void* ws, size_t ws_bytes, void* stream, int stages, int walk) {
  return gdn_fwd_impl(q, k, v, g, beta, h0, cu_seqlens, B, T, n_seqs, Hk, Hv, dk, dv, dtype, path, scale, o, hT, ws,
                      ws_bytes, stream, stages, walk);
}

extern "C" int rb2_gdn_bwd(const void* q, const void* k, const void* v, const float* g, const void* beta,
                           const float* h0, const int64_t* cu_seqlens, int64_t B, int64_t T, int64_t n_seqs,
                           int Hk, int Hv, int dk, int dv, int dtype, int path, float scale, const void* d_o,
                           const float* dhT, void* dq, void* dk_out, void* dv_out, float* dg, void* dbeta,
                           float* dh0, void* ws, size_t ws_bytes, void* stream) {
  return gdn_bwd_impl(q, k, v, g, beta, h0, cu_seqlens, B, T, n_seqs, Hk, Hv, dk, dv, dtype, path, scale, d_o, dhT,
                      dq, dk_out, dv_out, dg, dbeta, dh0, ws, ws_bytes, nullptr, 0, stream, 3, 0);
}

extern "C" int rb2_gdn_bwd_ex(const void* q, const void* k, const void* v, const float* g, const void* beta,
                              const float* h0, const int64_t* cu_seqlens, int64_t B, int64_t T, int64_t n_seqs,
                              int Hk, int Hv, int dk, int dv, int dtype, int path, float scale, const void* d_o,
                              const float* dhT, void* dq, void* dk_out, void* dv_out, float* dg, void* dbeta,
                              float* dh0, void* ws, size_t ws_bytes, void* scratch, size_t scratch_bytes,
                              void* stream, int stages, int walk) {
  return gdn_bwd_impl(q, k, v, g, beta, h0, cu_seqlens, B, T, n_seqs, Hk, Hv, dk, dv, dtype, path, scale, d_o, dhT,
                      dq, dk_out, dv_out, dg, dbeta, dh0, ws, ws_bytes, scratch, scratch_bytes, stream,
                      stages, walk);
}
