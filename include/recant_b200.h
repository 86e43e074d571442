/*
 * recant_b200 -- C ABI of the B200 (sm_100a) GDN + NVFP4 hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (as void*), launches
 * asynchronously on that stream, never allocates or frees device memory (scratch comes in as
 * `ws`/`ws_bytes`, sized by the matching *_workspace_size function) and returns a status code.
 * On a non-zero status, rb2_last_error() returns a message (thread-local).
 *
 * Layouts (all contiguous, row-major):
 *   q, k      [B*T, Hk, dk]     dtype RB2_F32 or RB2_BF16
 *   v         [B*T, Hv, dv]     same dtype
 *   g         [B*T, Hv]         float32 (log decay, <= 0)
 *   beta      [B*T, Hv]         same dtype as q
 *   o         [B*T, Hv, dv]     same dtype as q
 *   h0, hT    [N, Hv, dk, dv]   float32 (N = number of sequences)
 *   cu_seqlens int64 [N+1] on the DEVICE, or NULL for N = B fixed-length sequences of T
 * Hk must divide Hv (GQA: head h of v uses key/query head h / (Hv/Hk)); dk = dv = 128.
 */
#ifndef RECANT_B200_H
#define RECANT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RB2_API __attribute__((visibility("default")))
#else
#define RB2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define RB2_OK 0
#define RB2_EINVAL 1       /* bad argument: shape, dtype, null pointer, misalignment */
#define RB2_EUNSUPPORTED 2 /* valid but not implemented here (e.g. head dim != 128) */
#define RB2_ECUDA 3        /* a CUDA launch/runtime error */
#define RB2_EWORKSPACE 4   /* ws_bytes smaller than the *_workspace_size result */
#define RB2_ENOMEM 5       /* CUDA reported out of memory */
#define RB2_EDEVICE 6      /* a kernel reported an error through its device status word */

/* dtypes */
#define RB2_F32 0
#define RB2_BF16 1

/* GDN precision paths */
#define RB2_GDN_AUTO 0  /* bf16 inputs -> tensor-core path, f32 inputs -> exact fp32 path */
#define RB2_GDN_EXACT 1 /* fp32 CUDA-core arithmetic throughout (fp32 parity path) */
#define RB2_GDN_FAST 2  /* bf16 tensor-core path (bf16 inputs only) */

RB2_API const char* rb2_last_error(void);
RB2_API const char* rb2_version(void);

/* ---------------------------------------------------------------------------------------------
 * Chunked Gated DeltaNet.
 *
 * Replaces recant.model.ops.gdn_torch / gdn_fla as registered in GDN_BACKENDS
 * (recant/model/ops.py:21-60) and called by gdn_core (ops.py:62-67). Semantics are those of
 * gdn_torch: q and k are L2-normalised per head with eps 1e-6 inside the rsqrt (ops.py:18-19),
 * q is multiplied by `scale` (dk^-0.5 in the reference, ops.py:27), chunk size 64, state fp32.
 *
 * The forward stores everything the backward needs in `ws`; rb2_gdn_bwd must receive the same
 * `ws` contents and the same arguments. n_seqs = B without cu_seqlens, else len(cu_seqlens)-1
 * with B == 1.
 * ------------------------------------------------------------------------------------------- */
RB2_API size_t rb2_gdn_workspace_size(int64_t B, int64_t T, int64_t n_seqs, int Hk, int Hv, int dk, int dv,
                              int dtype, int path);

/* The workspace's two parts (no reference counterpart): `saved_bytes` is what the forward fills
 * and the backward reads -- the forward needs only this much -- and `scratch_bytes` is used only
 * inside the backward, which takes it either after the saved part of one buffer of
 * rb2_gdn_workspace_size bytes or as a separate buffer (rb2_gdn_bwd_ex), so one scratch buffer
 * can serve every layer of a model. Exact path: scratch 0. Returns a status code. */
RB2_API int rb2_gdn_workspace_split(int64_t B, int64_t T, int64_t n_seqs, int Hk, int Hv, int dk, int dv,
                                    int dtype, int path, size_t* saved_bytes, size_t* scratch_bytes);

RB2_API int rb2_gdn_fwd(const void* q, const void* k, const void* v, const float* g, const void* beta,
                const float* h0, const int64_t* cu_seqlens, int64_t B, int64_t T, int64_t n_seqs,
                int Hk, int Hv, int dk, int dv, int dtype, int path, float scale,
                void* o, float* hT, void* ws, size_t ws_bytes, void* stream);

/* Backward of rb2_gdn_fwd (the autograd of gdn_torch, ops.py:21-54): given dO (dtype) and
 * optionally dhT (fp32, NULL = zero), writes dq, dk [B*T,Hk,dk], dv [B*T,Hv,dv], dbeta (dtype),
 * dg (fp32) and, when dh0 != NULL, the gradient of the initial state (fp32). */
RB2_API int rb2_gdn_bwd(const void* q, const void* k, const void* v, const float* g, const void* beta,
                const float* h0, const int64_t* cu_seqlens, int64_t B, int64_t T, int64_t n_seqs,
                int Hk, int Hv, int dk, int dv, int dtype, int path, float scale,
                const void* d_o, const float* dhT, void* dq, void* dk_out, void* dv_out,
                float* dg, void* dbeta, float* dh0, void* ws, size_t ws_bytes, void* stream);

/* Stage-selecting forms of rb2_gdn_fwd / rb2_gdn_bwd for segmented and context-parallel runs
 * (no counterpart in the reference op; tensor-core path only). fwd stages: 1 = chunk table + per-
 * chunk prep, 2 = state walk, 3 = both. bwd stages: 1 = reversed state walk, 2 = chunk backward.
 * walk = 0: normal; 1: state only (final state / initial-state gradient, no per-chunk outputs);
 * 2 (fwd): transition -- U = 0 and S_0 = I for every sequence, so hT receives each sequence's
 * state-transition matrix M with S_out = M S_in + S_out(S_in = 0), and M^T maps the gradient of
 * the final state to that of the initial state. A later stage must see the same ws and arguments
 * (except h0 / dhT) as the stage-1 call that filled ws. bwd_ex's `scratch` (NULL = the part of ws
 * after the saved bytes) is the backward-only part of rb2_gdn_workspace_split. */
RB2_API int rb2_gdn_fwd_ex(const void* q, const void* k, const void* v, const float* g, const void* beta,
                           const float* h0, const int64_t* cu_seqlens, int64_t B, int64_t T, int64_t n_seqs,
                           int Hk, int Hv, int dk, int dv, int dtype, int path, float scale,
                           void* o, float* hT, void* ws, size_t ws_bytes, void* stream, int stages, int walk);
RB2_API int rb2_gdn_bwd_ex(const void* q, const void* k, const void* v, const float* g, const void* beta,
                           const float* h0, const int64_t* cu_seqlens, int64_t B, int64_t T, int64_t n_seqs,
                           int Hk, int Hv, int dk, int dv, int dtype, int path, float scale,
                           const void* d_o, const float* dhT, void* dq, void* dk_out, void* dv_out,
                           float* dg, void* dbeta, float* dh0, void* ws, size_t ws_bytes, void* scratch,
                           size_t scratch_bytes, void* stream, int stages, int walk);

/* Affine state fold of segmented / context-parallel GDN (no reference counterpart: the reference
 * walks one sequence's chunks in order, ops.py:49-52; a run of chunks maps S_out = M S_in + c and
 * dS_in = M^T dS_out + d). M, c: [n, H, d, d] fp32 (c NULL = 0); s0: [H, d, d] (NULL = zero, or
 * the identity when identity_init). transpose = 0: x_0 = s0, x_{k+1} = M_k x_k + c_k; transpose
 * = 1: from k = n-1 down to 0, x <- M_k^T x + c_k. states (optional, [n, H, d, d]) receives the
 * value entering every map, final_out (optional, [H, d, d]) the value after the last. d = 128;
 * pointers 16-byte aligned; n may be 0 (final_out = s0). */
RB2_API int rb2_gdn_state_fold(const float* M, const float* c, const float* s0, int64_t n, int H, int d,
                               int transpose, int identity_init, float* states, float* final_out, void* stream);

/* rb2_gdn_state_fold with a prefix run and an explicit mode. mode 0: ascending k, x <- M_k x + c_k;
 * mode 1: descending k, x <- M_k^T x + c_k (= transpose 1); mode 2: ascending k, x <- M_k^T x + c_k
 * (pass transposed maps G_k = M_k^T to apply M_k: the fastest form). The np maps (Mp, cp) are applied
 * first, in the same mode and order, their entering values not recorded; states records the values
 * entering the n main maps. */
RB2_API int rb2_gdn_state_fold_ex(const float* M, const float* c, int64_t n, const float* Mp, const float* cp,
                                  int64_t np, const float* s0, int H, int d, int mode, int identity_init,
                                  float* states, float* final_out, void* stream);

/* Recurrent (token-by-token) forward for short calls with a carried state: the decode step of
 * GatedDeltaNet.forward with a LayerCache (layers.py:177-180; serve/engine.py:107-119), the same
 * arithmetic as gdn_torch on one padded chunk (ops.py:21-54). Arguments as rb2_gdn_fwd without
 * path / workspace; no backward (the serving path runs under no_grad). h0, hT: [n_seqs, Hv, 128,
 * 128] fp32, either may be NULL, hT may equal h0 (updated in place). Cost: one read and one write
 * of the state per call, O(T) sequential steps. */
RB2_API int rb2_gdn_recurrent_fwd(const void* q, const void* k, const void* v, const float* g, const void* beta,
                                  const float* h0, const int64_t* cu_seqlens, int B, int T, int n_seqs, int Hk,
                                  int Hv, int dk, int dv, int dtype, float scale, void* o, float* hT, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Element-wise stages of the GDN block (recant/model/layers.py:148-182), bf16 activations:
 *
 * rb2_conv_silu_fwd: y = silu(bf16(causal depthwise conv1d(x, w))), x [B, T, C], w [C, K] (K = 4,
 *   zero prefix; layers.py:157-168). The output channels go to y0 (all C when y1 = y2 = NULL) or are
 *   split into y0 [B, T, s1], y1 [B, T, s2 - s1], y2 [B, T, C - s2] -- the block's q, k, v
 *   (layers.py:169). prev (NULL = zeros) is the cached prefix [B, C, 3] of the decode path
 *   (LayerCache.conv_state: token -3 + j in column j, layers.py:159-166); new_state (optional,
 *   [B, C, 3]) receives the last 3 tokens of cat(prev, x), the next call's prefix; it may be prev
 *   itself (updated in place).
 *   rb2_conv_silu_bwd: dx from x, prev, w and the output gradient (same split; prev gets no gradient,
 *   as the reference's cache is detached).
 * rb2_gdn_gates_fwd: g = -exp(A_log[h]) softplus(a + dt_bias[h]) (fp32) and beta = sigmoid(b)
 *   (bf16) over n = B*T*H entries (fused_ops.py:32-33, layers.py:154); _bwd gives da, db.
 * rb2_gated_rmsnorm_fwd: per row of dim = 128, y = bf16(w * bf16(x rsqrt(mean x^2 + eps))) *
 *   silu(z) (fused_ops.py:11-16), rstd [rows] saved for rb2_gated_rmsnorm_bwd (dx, dz).
 * The block's conv, gate and norm weights are frozen (the reference trains LoRA only), so only
 * input gradients are produced.
 * ------------------------------------------------------------------------------------------- */
RB2_API int rb2_conv_silu_fwd(const void* x, const void* w, const void* prev, int B, int T, int C, int K, void* y0,
                              void* y1, void* y2, int s1, int s2, void* new_state, void* stream);
RB2_API int rb2_conv_silu_bwd(const void* x, const void* w, const void* prev, const void* dy0, const void* dy1,
                              const void* dy2, int s1, int s2, int B, int T, int C, int K, void* dx, void* stream);
RB2_API int rb2_gdn_gates_fwd(const void* a, const void* b, const float* A_log, const float* dt_bias, int64_t n,
                              int H, float* g, void* beta, void* stream);
RB2_API int rb2_gdn_gates_bwd(const void* a, const void* beta, const float* A_log, const float* dt_bias,
                              const float* dg, const void* dbeta, int64_t n, int H, void* da, void* db, void* stream);
RB2_API int rb2_gated_rmsnorm_fwd(const void* x, const void* z, const float* w, int64_t rows, int dim, float eps,
                                  void* y, float* rstd, void* stream);
RB2_API int rb2_gated_rmsnorm_bwd(const void* x, const void* z, const float* w, const float* rstd, const void* dout,
                                  int64_t rows, int dim, void* dx, void* dz, void* stream);

/* ---------------------------------------------------------------------------------------------
 * NVFP4 quantizer: codes/scales/gscale of quantize(rht(x)) (use_rht=1) or quantize(x),
 * bit-exact with recant/model/nvfp4.py:23-31,59-91 for round-to-nearest; stochastic=1 is the
 * unbiased rounding of nvfp4.py:62-68 driven by a Philox-4x32-10 stream keyed by `seed`.
 * Replaces nvfp4.quantize_activation's fast hook (nvfp4.py:139-149, fp4_kernels.quantize_fast
 * at recant/model/fp4_kernels.py:452-467). x [M,K] with K % 16 == 0, dtype F32 or BF16.
 * Outputs: codes u8 [M, K/2] (even element in the low nibble), scales e4m3 bytes [M, K/16],
 * optional scales_blocked (the 128x4 blocked swizzle of nvfp4._to_blocked, nvfp4.py:112-119,
 * ceil(M/128)*ceil(K/64)*512 bytes, pad bytes zero) and gscale (1 float, device).
 * ------------------------------------------------------------------------------------------- */
RB2_API size_t rb2_nvfp4_quantize_workspace_size(int64_t M, int64_t K);

RB2_API int rb2_nvfp4_quantize(const void* x, int64_t M, int64_t K, int dtype, int use_rht, int stochastic,
                       uint64_t seed, uint8_t* codes, uint8_t* scales, uint8_t* scales_blocked,
                       float* gscale, void* ws, size_t ws_bytes, void* stream);

/* Allocation-free rb2_nvfp4_quantize (no counterpart in the reference). For callers that cannot
 * provide device scratch -- C/C++ embedders without a device allocator, serving loops whose
 * allocator is frozen, code where a cudaMalloc would synchronise or break a memory cap -- the
 * quantizer's one scratch word (the global |x| maximum) lives in a 256-byte file-scope device
 * array that every GPU loading the library keeps until exit. Same arguments and results as
 * rb2_nvfp4_quantize minus ws/ws_bytes. The scratch is one word for every shape, so no size is
 * rejected today (RB2_EWORKSPACE stays as a guard should a shape ever need more than the 256-byte
 * array). The first call on each device, and the first after that device's context is replaced
 * (e.g. by cudaDeviceReset), looks the array's address up; make that call before any stream
 * capture. All calls share the array and each call clears the word first; calls that overlap on
 * the GPU (concurrent streams) race on it. Never allocates or frees device memory. */
RB2_API int rb2_nvfp4_quantize_noalloc(const void* x, int64_t M, int64_t K, int dtype, int use_rht, int stochastic,
                                       uint64_t seed, uint8_t* codes, uint8_t* scales, uint8_t* scales_blocked,
                                       float* gscale, void* stream);

/* Gated RMSNorm (as rb2_gated_rmsnorm_fwd) fused with the NVFP4 quantize of its output: y = the
 * norm of x gated by z (fused_ops.py:11-16) and rstd as rb2_gated_rmsnorm_fwd, plus codes / scales /
 * blocked scales / gscale of quantize(rht(y)) (RN) as rb2_nvfp4_quantize on y viewed as [M, K]
 * (rows * 128 == M * K) -- the out_proj input of GatedDeltaNet.forward (layers.py:181, QLinear ->
 * quantize_activation, nvfp4.py:144-149). The global amax is reduced in the norm's own pass, so y
 * is read once more (by the code pass) instead of twice. ws: rb2_nvfp4_quantize_workspace_size(M, K). */
RB2_API int rb2_gated_rmsnorm_nvfp4_fwd(const void* x, const void* z, const float* w, int64_t rows, int dim, float eps,
                                        void* y, float* rstd, int64_t M, int64_t K, int use_rht, uint8_t* codes,
                                        uint8_t* scales, uint8_t* scales_blocked, float* gscale, void* ws,
                                        size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Narrow bf16 projection: out[M,N] = A[M,K] . B[N,K]^T, fp32 accumulation, out bf16 (RB2_BF16) or
 * fp32 (RB2_F32) with row stride ldo. Replaces the block's dense projections that are too narrow for
 * NVFP4 -- in_proj_b / in_proj_a (recant/model/layers.py:154-155; QLinear keeps N < 256 unquantized,
 * layers.py:47-48) -- and the LoRA down-projections x A^T (layers.py:65-69, 86-88), concatenated
 * along N so that one pass over x yields all of them. B contiguous [N][K]; A row stride lda
 * (elements). Needs 16 <= N <= 256 with N % 16 == 0, K % 64 == 0, lda and ldo multiples of 8, A, B
 * and out 16-byte aligned. */
RB2_API int rb2_skinny_gemm(const void* A, int64_t lda, const void* B, int64_t M, int64_t N, int64_t K, void* out,
                            int64_t ldo, int out_dtype, void* stream);

/* ---------------------------------------------------------------------------------------------
 * LoRA up-projection added to a base output: out[m, n] = y[m, n] + s * sum_k h[m, k] B[n, k] over
 * k < r (1 <= r <= 128), fp32 accumulation, rounded as the reference's ops round it on the GPU --
 * mode 0: grouped_linear's torch.addmm(y, h, B^T, alpha=s) (recant/model/layers.py:86-97), which
 * cuBLAS computes as bf16(y + bf16(s * acc)); mode 1: QLinear.forward's y + (h B^T) * s
 * (layers.py:65-70), the product, its scaling and the sum each rounded to bf16. y, h, B, out bf16 with row strides ldy, ldh, ldb, ldo (multiples
 * of 8 elements, 16-byte aligned bases; h's and B's columns past r are not read); out may be y. ws:
 * rb2_lora_up_workspace_size() bytes (the op's status word, cleared by the call). */
RB2_API size_t rb2_lora_up_workspace_size(void);
RB2_API int rb2_lora_up(const void* y, int64_t ldy, const void* h, int64_t ldh, const void* B, int64_t ldb, int64_t M,
                        int64_t N, int r, float scale, int mode, void* out, int64_t ldo, void* ws, size_t ws_bytes,
                        void* stream);

/* ---------------------------------------------------------------------------------------------
 * LoRA weight gradient: out(n, r) = bf16(bf16(sum_m D[m, n] H[m, r]) * scale) as fp32, for
 * n < N, r < R, the sum over the M tokens. Replaces the cuBLAS products that torch's autograd runs
 * for the gradients of the block's fp32 LoRA factors (recant/model/layers.py:65-70, 86-97): for
 * dB = s dy^T h (the mat2 gradient of grouped_linear's addmm(y, h, B^T, alpha=s), or of QLinear's
 * (h B^T) * s) pass D = dy [M, out], H = h [M, r], scale = s; for dA = (x^T dh)^T (the gradient of
 * x A^T) pass D = x [M, in], H = dh [M, r], scale = 1. The roundings are the reference's: the bf16
 * product, the bf16 multiply by alpha, and the cast back to the fp32 parameter; only the order of
 * the fp32 sum over tokens differs. D, H bf16 with row strides ldd, ldh (multiples of 8 elements,
 * 16-byte aligned bases; H's columns past R are not read); 1 <= R <= 64. out fp32 at
 * out[n * ld_n + r * ld_r], either [N, R] (ld_r = 1) or [R, N] (ld_n = 1). M = 0 writes zeros (D and H
 * may then be NULL).
 * ws: rb2_lora_wgrad_workspace_size(M, N, R) bytes, 256-byte aligned; its first 4 bytes are the
 * op's status word (cleared by the call). Deterministic: the token splits are summed in a fixed
 * order. */
RB2_API size_t rb2_lora_wgrad_workspace_size(int64_t M, int64_t N, int R);
RB2_API int rb2_lora_wgrad(const void* D, int64_t ldd, const void* H, int64_t ldh, int64_t M, int64_t N, int R,
                           float scale, float* out, int64_t ld_n, int64_t ld_r, void* ws, size_t ws_bytes,
                           void* stream);

/* Scale bytes [rows, cols] (e4m3) -> the 128x4 blocked swizzle of nvfp4._to_blocked
 * (recant/model/nvfp4.py:112-119), ceil(rows/128)*ceil(cols/4)*512 bytes, pad bytes zero. Lets
 * FP4 tensors quantized elsewhere (e.g. by the reference's quantize_weight) feed the GEMM. */
RB2_API int rb2_nvfp4_block_scales(const uint8_t* scales, int64_t rows, int64_t cols, uint8_t* blocked, void* stream);

/* ---------------------------------------------------------------------------------------------
 * NVFP4 block-scaled GEMM: out[M,N] = (A . B^T) * gA * gB where A = codes_a [M,K/2] with
 * blocked scales (128x4 swizzle) and B = codes_b [N,K/2] likewise; fp32 accumulation.
 * Replaces the GEMM_BACKENDS entries of recant/model/nvfp4.py:108-125 (_gemm_emulated and
 * _gemm_scaled_mm = torch._scaled_mm on cuBLASLt). out_dtype RB2_F32 or RB2_BF16.
 * Requires K % 64 == 0.
 * ------------------------------------------------------------------------------------------- */
RB2_API size_t rb2_nvfp4_gemm_workspace_size(int64_t M, int64_t N, int64_t K);

RB2_API int rb2_nvfp4_gemm(const uint8_t* a_codes, const uint8_t* a_scales_blocked, const float* a_gscale,
                   const uint8_t* b_codes, const uint8_t* b_scales_blocked, const float* b_gscale,
                   int64_t M, int64_t N, int64_t K, void* out, int out_dtype, void* ws,
                   size_t ws_bytes, void* stream);
/* rb2_nvfp4_gemm with two optional extras (no reference counterpart for the first; the second is
 * the "lora?" of the GEMM boundary):
 * - b_images: B's scales as the kernel reads them, prepared by rb2_nvfp4_gemm_b_images for frozen
 *   weights (NULL = read b_scales_blocked). The kernel reads the 128x4 blocked layout in place
 *   (one 512-byte atom per 128-row block and 64-element K step), so these are a copy of B's
 *   blocked scales: 16-byte aligned, rb2_nvfp4_gemm_b_images_size(N, K) bytes.
 * - lora_h (NULL = none): out = a . b^T * gA * gB + lora_scale * lora_h . lora_b^T with lora_h
 *   [M, lora_r] bf16 (row stride lora_ldh elements) and lora_b [N, lora_r] bf16, lora_r 8 or 16:
 *   QLinear's LoRA y + (alpha / r) (x A^T) B^T (layers.py:65-70, 86-97) with h = x A^T computed by
 *   the caller. fp32 output: one fp32 sum. bf16 output, rounded as the reference's ops round on
 *   the GPU: lora_mode 0 = grouped_linear's addmm (y to bf16, s h B^T to bf16, their sum rounded);
 *   lora_mode 1 = QLinear.forward's three ops (y, h B^T and s h B^T each to bf16, then the sum). */
RB2_API int rb2_nvfp4_gemm_ex(const uint8_t* a_codes, const uint8_t* a_scales_blocked, const float* a_gscale,
                              const uint8_t* b_codes, const uint8_t* b_scales_blocked, const float* b_gscale,
                              const uint8_t* b_images, const void* lora_h, int64_t lora_ldh, const void* lora_b,
                              int lora_r, float lora_scale, int lora_mode, int64_t M, int64_t N, int64_t K, void* out,
                              int out_dtype, void* ws, size_t ws_bytes, void* stream);
/* rb2_nvfp4_gemm on SM pairs: two-CTA clusters (tcgen05 cta_group::2) computing 256 x 256 tiles, each
 * CTA holding its own 128 rows of A and half of B's 256 rows (no multicast loads). Same arguments,
 * layouts and results as rb2_nvfp4_gemm (no LoRA, no b_images); an alternative kept for measurement:
 * at 16384 x 12288 x 4096 it takes 0.56 ms against rb2_nvfp4_gemm's 0.46 ms. */
RB2_API int rb2_nvfp4_gemm_pair(const uint8_t* a_codes, const uint8_t* a_scales_blocked, const float* a_gscale,
                                const uint8_t* b_codes, const uint8_t* b_scales_blocked, const float* b_gscale,
                                int64_t M, int64_t N, int64_t K, void* out, int out_dtype, void* ws,
                                size_t ws_bytes, void* stream);
/* rb2_nvfp4_gemm for M <= 4 rows of A (the decode step: one token per sequence; no counterpart in
 * the reference, whose GEMM backends serve every M alike, nvfp4.py:108-125): reads each row of B
 * once, one warp per row, instead of 128-row tensor-core tiles. Scales are the row-major e4m3 bytes
 * [rows, K/16] (FP4Tensor.scales), not the blocked layout. K % 32 == 0, M x K within shared memory
 * (about 12k columns at M = 4); out [M, N] fp32 or bf16. */
RB2_API int rb2_nvfp4_gemv(const uint8_t* a_codes, const uint8_t* a_scales, const float* a_gscale,
                           const uint8_t* b_codes, const uint8_t* b_scales, const float* b_gscale, int64_t M,
                           int64_t N, int64_t K, void* out, int out_dtype, void* stream);
RB2_API size_t rb2_nvfp4_gemm_b_images_size(int64_t N, int64_t K);
RB2_API int rb2_nvfp4_gemm_b_images(const uint8_t* b_scales_blocked, int64_t N, int64_t K, void* out,
                                    size_t out_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Launch profiler (no counterpart in the reference; measurement support for benchmarks).
 * While enabled, each kernel launch of this library is bracketed by CUDA events on its stream.
 * rb2_profile_read waits for them and writes up to max_records (name, milliseconds) pairs; names
 * are NUL-terminated in slots of name_stride bytes. Not thread-safe.
 * ------------------------------------------------------------------------------------------- */
RB2_API int rb2_profile_enable(int max_launches);
RB2_API int rb2_profile_disable(void);
RB2_API int rb2_profile_read(int max_records, char* names, size_t name_stride, float* ms);
RB2_API int rb2_profile_dropped(void);

/* ---------------------------------------------------------------------------------------------
 * Device status words (the reference's wrapper contract: device-side guards write an error word
 * that the wrapper checks). Every mbarrier wait in this library's kernels is bounded: when one runs
 * out (a load or a product that never completes), the kernel records a nonzero code in its op's
 * status word, skips the rest of its work and returns, so the context stays usable. The word is the
 * first 4 bytes of the op's workspace for rb2_gdn_fwd / rb2_gdn_bwd (of the saved part, with
 * rb2_gdn_workspace_split), rb2_nvfp4_gemm / _ex / _pair; the operation clears it when it starts
 * (the GDN forward; the GEMM calls). rb2_skinny_gemm keeps its word in the library.
 * ------------------------------------------------------------------------------------------- */
/* Synchronises `stream`, copies the status word at device address `status_word` to *code and, with
 * `clear`, zeroes it. */
RB2_API int rb2_status_read(const void* status_word, int* code, int clear, void* stream);
/* rb2_skinny_gemm's status word (synchronises the device; `clear` zeroes it). */
RB2_API int rb2_skinny_gemm_status(int* code, int clear);
/* Self-test of the bounded wait: one kernel waits on an mbarrier that one arrival completed (it must
 * return at once; if not, code 902) and then on one that nothing completes, which must give up after
 * `max_polls` polls (0 < max_polls <= 2^24; 2^14 polls take well under a millisecond) and record 901
 * in the device int `*status`. Afterwards the context is usable as before. */
RB2_API int rb2_selftest_wait(int* status, unsigned int max_polls, void* stream);

/* Diagnostic (no counterpart in the reference): one-tile tcgen05 product D[M,N] = A . B^T with
 * bf16 A, B given K-major (a_mn/b_mn = 0: A[m*K+k]) or MN-major (1: A[k*M+m]); M in {64,128},
 * N, K in {64,128}; fp32 D. Validates the tensor-core operand layouts on this device. */
RB2_API int rb2_selftest_mma(const void* A, const void* B, float* D, int a_mn, int b_mn, int M, int N, int K,
                             int* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RECANT_B200_H */
