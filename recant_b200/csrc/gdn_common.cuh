// Shared pieces of the chunked GDN kernels: problem description, chunk table, workspace layout.
#pragma once

#include "common.cuh"

namespace rb2 {

constexpr int kChunk = 64;   // chunk length C (recant/model/ops.py:21 chunk_size=64)
constexpr int kHead = 128;   // dk = dv

struct GdnProblem {
  const void* q; const void* k; const void* v; const float* g; const void* beta;
  const float* h0; const int64_t* cu_seqlens;
  int64_t B, T, n_seqs, tokens;
  int Hk, Hv, group;           // group = Hv / Hk
  int dtype, path;
  float scale;
  int max_chunks;              // bound on the chunk count: tokens/64 + n_seqs
  int stages = 3;              // fwd: 1 = chunk table + prep, 2 = state walk; bwd: 1 = walk, 2 = chunks
  int walk = 0;                // 0 normal; 1 state only (no per-chunk outputs); 2 transition (fwd):
                               // U = 0 and S_0 = I, so the final "state" is the segment's matrix M
};

// Chunk table built on the device from cu_seqlens (or from B, T): chunk ci covers tokens
// [tok0[ci], tok0[ci] + len[ci]) of sequence seq[ci]; sequence s owns chunks
// [seq_chunk0[s], seq_chunk0[s+1]).
struct ChunkTable {
  int* tok0; int* len; int* seq; int* seq_chunk0; int* n_chunks;
  int* order;  // [n_seqs] sequences longest first (ties: lower index); the walks take them in this order
};

// fp32 workspace of the exact path; every per-(chunk, head) array is indexed by ch = ci*Hv + h.
struct ExactWs {
  int* err;       // the op's device status word, the first 4 bytes of the (saved) workspace: 0 here
  ChunkTable ct;
  float* stats;   // [ch][4][64]: cum, rq, rk, beta
  float* qn;      // [ch][64][128]  q * rsqrt(|q|^2 + eps) * scale
  float* kn;      // [ch][64][128]  k * rsqrt(|k|^2 + eps)
  float* tinv;    // [ch][64][64]   (I + strict_lower(beta k k^T * Gamma))^-1
  float* aqk;     // [ch][64][64]   (q k^T) * Gamma, lower incl. diagonal
  float* u;       // [ch][64][128]
  float* w;       // [ch][64][128]
  float* hs;      // [ch][128][128] state entering the chunk
  float* vp;      // [ch][64][128]  V' = U - W S
  // backward
  float* dh;      // [ch][128][128] gradient of the state leaving the chunk
  float* dvp;     // [ch][64][128]
  float* dqt;     // [ch][64][128]
  float* dw;      // [ch][64][128]
  float* dkt;     // [ch][64][128]
  float* daqk;    // [ch][64][64]
  float* dgam;    // [ch]
  float* dqh;     // [tokens][Hv][128] per-value-head dq (GQA only)
  float* dkh;     // [tokens][Hv][128]
};

inline int gdn_max_chunks(int64_t tokens, int64_t n_seqs) {
  return int(tokens / kChunk + n_seqs);
}

template <typename Ws>
size_t carve_exact(Carver& c, Ws& w, int64_t tokens, int64_t n_seqs, int Hv, int max_chunks, bool gqa) {
  const size_t nch = size_t(max_chunks) * Hv;
  w.err = c.template take<int>(1);  // first: every GDN workspace starts with its status word
  w.ct.tok0 = c.template take<int>(max_chunks);
  w.ct.len = c.template take<int>(max_chunks);
  w.ct.seq = c.template take<int>(max_chunks);
  w.ct.seq_chunk0 = c.template take<int>(n_seqs + 1);
  w.ct.order = c.template take<int>(n_seqs);
  w.ct.n_chunks = c.template take<int>(1);
  w.stats = c.template take<float>(nch * 4 * 64);
  w.qn = c.template take<float>(nch * 64 * 128);
  w.kn = c.template take<float>(nch * 64 * 128);
  w.tinv = c.template take<float>(nch * 64 * 64);
  w.aqk = c.template take<float>(nch * 64 * 64);
  w.u = c.template take<float>(nch * 64 * 128);
  w.w = c.template take<float>(nch * 64 * 128);
  w.hs = c.template take<float>(nch * 128 * 128);
  w.vp = c.template take<float>(nch * 64 * 128);
  w.dh = c.template take<float>(nch * 128 * 128);
  w.dvp = c.template take<float>(nch * 64 * 128);
  w.dqt = c.template take<float>(nch * 64 * 128);
  w.dw = c.template take<float>(nch * 64 * 128);
  w.dkt = c.template take<float>(nch * 64 * 128);
  w.daqk = c.template take<float>(nch * 64 * 64);
  w.dgam = c.template take<float>(nch);
  w.dqh = c.template take<float>(gqa ? size_t(tokens) * Hv * 128 : 0);
  w.dkh = c.template take<float>(gqa ? size_t(tokens) * Hv * 128 : 0);
  return c.bytes();
}

// Launch the chunk-table builder (one CTA). Defined in gdn_exact.cu.
int launch_chunk_table(const GdnProblem& p, const ChunkTable& ct, cudaStream_t s);

}  // namespace rb2
