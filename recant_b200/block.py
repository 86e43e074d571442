"""The GDN block on B200: recant/model/layers.py:148-182 (``GatedDeltaNet``) with the reference's
parameter names, built from this package's kernels.

x [B, T, hidden] bf16 ->
  qkv, z      = NVFP4 in_proj_qkv / in_proj_z (+ LoRA), one shared activation quantize
                (layers.py:152, grouped_linear layers.py:72-97; QLinear layers.py:36-70)
  beta, a     = sigmoid(in_proj_b(x)), in_proj_a(x): bf16 dense, N = Hv < 256, never quantized
                (layers.py:154-155, 47-48)
  conv        = silu(causal depthwise conv1d, kernel 4; zero prefix, or the cached one when a
                LayerCache is given, which then receives the next prefix)  (layers.py:157-168)
  q, k, v     = split(conv) into [Hk*128, Hk*128, Hv*128]                  (layers.py:169-172)
  g           = -exp(A_log) softplus(a + dt_bias)                          (fused_ops.py:32-33)
  core        = GDN (``gdn_b200``; Hk < Hv handled without repeat_interleave); with a cache the
                recurrent state is carried in and out (layers.py:177-180): short calls take the
                token-by-token kernel, longer ones the chunked op
  y           = out_proj(RMSNormGated(core, z))  (NVFP4 + LoRA)            (layers.py:23-34,181)

Kernels: ``rb2_conv_silu_*``, ``rb2_gdn_gates_*``, ``rb2_gated_rmsnorm_*`` (csrc/gdn_block.cu), the
NVFP4 quantizer and GEMM, the GDN op, and ``rb2_skinny_gemm`` (csrc/skinny_gemm.cu) for the narrow
projections of x: in_proj_b, in_proj_a and the LoRA down-projections of in_proj_qkv / in_proj_z
come from one pass over x (:class:`_XProjections`). The LoRA up-projections and the LoRA weight
gradients are plain GEMMs through torch (cuBLAS). Frozen weights get no gradients; LoRA A and B do.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn

from . import _lib as L
from . import nvfp4 as N
from .gdn import RECURRENT_MAX_T, _stream, gdn_b200, gdn_recurrent


def _p(t):
    return L.ptr(t)


# The gated norm reduces out_proj's quantizer amax in its own pass (rb2_gated_rmsnorm_nvfp4_fwd) when
# y has more blocks of 16 than the quantizer's single-launch limit; smaller calls (the decode step)
# keep the norm and the one-launch quantizer.
FUSE_NORM_QUANT = True
NORM_QUANT_MIN_BLOCKS = 2048

# The narrow projections of x run on rb2_skinny_gemm from this many rows on; shorter calls (the
# decode step's few rows) keep the cuBLAS GEMV-like path, which has less latency for one tile.
NARROW_MIN_ROWS = 65


def narrow_product(x2, w):
    """x2 [M, K] bf16 . w [N, K]^T bf16 -> bf16 [M, N] on the library's tcgen05 kernel (N <= 256, K a
    multiple of 64; N is padded to a multiple of 16 with zero rows)."""
    M, K = x2.shape
    n = w.shape[0]
    npad = -(-n // 16) * 16
    if npad != n:
        w = torch.cat([w, w.new_zeros(npad - n, K)], 0)
    w = w.contiguous()
    out = torch.empty(M, npad, dtype=torch.bfloat16, device=x2.device)
    L.check(L.lib().rb2_skinny_gemm(_p(x2), x2.stride(0), _p(w), M, npad, K, _p(out), npad, L.BF16,
                                    _stream(x2.device)), "skinny_gemm")
    L.check_skinny_status()
    return out[:, :n]


def _wgrad_ok(d2, h):
    """Both operands as rb2_lora_wgrad reads them: CUDA bf16 rows (unit column stride, row strides
    multiples of 8 elements, 16-byte aligned) and a rank of at most 64."""
    return (d2.is_cuda and d2.dtype == torch.bfloat16 and h.dtype == torch.bfloat16 and d2.dim() == 2 and h.dim() == 2
            and d2.shape[0] == h.shape[0] and 1 <= h.shape[1] <= 64 and d2.shape[1] >= 1
            and d2.stride(1) == 1 and h.stride(1) == 1 and d2.stride(0) % 8 == 0 and h.stride(0) % 8 == 0
            and d2.stride(0) >= d2.shape[1] and h.stride(0) >= h.shape[1]
            and d2.data_ptr() % 16 == 0 and h.data_ptr() % 16 == 0)


def lora_wgrad(d2, h, scale=1.0, transposed=False):
    """fp32 LoRA factor gradient from the library's tcgen05 kernel: out[n, r] = bf16(bf16(d2^T h) * scale)
    over the M rows of d2 [M, N] and h [M, R] (bf16), as [N, R], or [R, N] with ``transposed`` --
    the gradients torch's autograd gives the fp32 factors through their bf16 casts (dB = s dy^T h for
    h B^T; dA = (x^T dh)^T for x A^T; layers.py:65-70, 86-97)."""
    if not _wgrad_ok(d2, h):
        raise ValueError("recant_b200.lora_wgrad: needs CUDA bf16 [M, N] and [M, R <= 64] rows with unit column "
                         "stride, row strides a multiple of 8 elements and 16-byte aligned bases")
    M, n = d2.shape
    R = h.shape[1]
    out = torch.empty((R, n) if transposed else (n, R), dtype=torch.float32, device=d2.device)
    ws = torch.empty(L.lib().rb2_lora_wgrad_workspace_size(M, n, R), dtype=torch.uint8, device=d2.device)
    ld_n, ld_r = (1, n) if transposed else (R, 1)
    L.check(L.lib().rb2_lora_wgrad(_p(d2), d2.stride(0), _p(h), h.stride(0), M, n, R, float(scale), _p(out), ld_n,
                                   ld_r, _p(ws), ws.numel(), _stream(d2.device)), "lora_wgrad")
    L.check_status(ws, "lora_wgrad")
    return out


# rb2_lora_up takes products of at least this many rows; shorter ones (the decode step's few tokens)
# keep the reference's torch ops, which cost less than a 128-row tile per 128 output columns there
# (B=1 graphed decode step: 0.125 ms with the kernel, 0.109 ms without).
LORA_UP_MIN_ROWS = 65


def _up_ok(y2, h, b):
    """Operands as rb2_lora_up reads them: CUDA bf16 rows with unit column stride, row strides
    multiples of 8 elements, 16-byte aligned bases, rank at most 128."""
    ts = (y2, h, b)
    return (all(t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 2 and t.stride(1) == 1 and t.stride(0) % 8 == 0
                and t.stride(0) >= t.shape[1] and t.data_ptr() % 16 == 0 for t in ts)
            and h.shape[0] == y2.shape[0] and b.shape[0] == y2.shape[1] and h.shape[1] == b.shape[1]
            and 1 <= h.shape[1] <= 128)


def _use_up(y2, h, b):
    """Whether the block takes rb2_lora_up for this product: switched on, enough rows, operands fit."""
    return LORA_UP and y2.dim() == 2 and y2.shape[0] >= LORA_UP_MIN_ROWS and _up_ok(y2, h, b)


def lora_up(y2, h, b, scale, mode):
    """y2 + scale (h b^T) on the library's tcgen05 kernel, rounded as the reference's ops round it on
    the GPU: ``mode`` 0 as torch.addmm(y2, h, b^T, alpha=scale) (layers.py:86-97; cuBLAS rounds the
    scaled product to bf16, then adds), 1 as QLinear's three bf16 ops (layers.py:65-70);
    y2 [M, N], h [M, r], b [N, r] bf16, r <= 128. Returns a new [M, N] bf16 tensor."""
    if not _up_ok(y2, h, b):
        raise ValueError("recant_b200.lora_up: needs CUDA bf16 [M, N], [M, r], [N, r] rows (r <= 128) with unit "
                         "column stride, row strides a multiple of 8 elements and 16-byte aligned bases")
    M, n = y2.shape
    out = torch.empty(M, n, dtype=torch.bfloat16, device=y2.device)
    ws = torch.empty(L.lib().rb2_lora_up_workspace_size(), dtype=torch.uint8, device=y2.device)
    L.check(L.lib().rb2_lora_up(_p(y2), y2.stride(0), _p(h), h.stride(0), _p(b), b.stride(0), M, n, h.shape[1],
                                float(scale), int(mode), _p(out), n, _p(ws), ws.numel(), _stream(y2.device)),
            "lora_up")
    L.check_status(ws, "lora_up")
    return out


def _pow2(s):
    """Whether scaling by s is exact in binary floating point (s a power of two)."""
    return s > 0 and math.frexp(s)[0] == 0.5


# The LoRA up-projection (y + s h B^T) runs on rb2_lora_up; off, as the reference's torch ops.
LORA_UP = True

# The LoRA factor gradients (dA, dB) run on rb2_lora_wgrad; off, torch's autograd computes them with
# cuBLAS as the reference does.
LORA_WGRAD = True


def _narrow_ok(x, n):
    x2_rows = x.numel() // x.shape[-1]
    return (x.is_cuda and x.dtype == torch.bfloat16 and x.shape[-1] % 64 == 0 and 0 < n <= 256
            and x2_rows >= NARROW_MIN_ROWS)


class _XProjections(torch.autograd.Function):
    """The block's narrow projections of x in one pass: [x W_f^T | x A_1^T | x A_2^T ...] with W_f the
    frozen bf16 rows (in_proj_b, in_proj_a; layers.py:154-155) and A_i the LoRA down-projection
    weights of the grouped in_proj (layers.py:86-88, cast to bf16 as the reference casts them).
    Backward: dx = dout . [W_f; A_i] and dA_i = (dh_i^T x) in bf16 then fp32, the gradient the
    reference's autograd gives through ``A.to(x.dtype)``; W_f gets none."""

    @staticmethod
    def forward(ctx, x, w_frozen, *As):
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
            x2 = x2.contiguous()
        W = torch.cat([w_frozen.to(torch.bfloat16)] + [a.to(torch.bfloat16) for a in As], 0).contiguous()
        out = narrow_product(x2, W)
        ctx.save_for_backward(x2, W)
        ctx.n_frozen = w_frozen.shape[0]
        ctx.ranks = [a.shape[0] for a in As]
        ctx.xshape = x.shape
        return out.reshape(*x.shape[:-1], W.shape[0])

    @staticmethod
    def backward(ctx, dout):
        x2, W = ctx.saved_tensors
        d2 = dout.reshape(-1, dout.shape[-1]).to(torch.bfloat16)
        dx = (d2 @ W).reshape(ctx.xshape) if ctx.needs_input_grad[0] else None
        grads, off = [], ctx.n_frozen
        need = [ctx.needs_input_grad[2 + i] for i in range(len(ctx.ranks))]
        dh_all = d2[:, off:off + sum(ctx.ranks)]
        if LORA_WGRAD and any(need) and _wgrad_ok(x2, dh_all):
            dA = lora_wgrad(x2, dh_all, 1.0, transposed=True)  # every member's dA in one pass over x
            for i, r in enumerate(ctx.ranks):
                grads.append(dA[off - ctx.n_frozen:off - ctx.n_frozen + r] if need[i] else None)
                off += r
            return (dx, None, *grads)
        for i, r in enumerate(ctx.ranks):
            grads.append((d2[:, off:off + r].t() @ x2).float() if need[i] else None)
            off += r
        return (dx, None, *grads)


class _InProj(torch.autograd.Function):
    """The block's input projections of x as one function (layers.py:86-97, 154-155): the NVFP4
    products of in_proj_qkv / in_proj_z from one activation quantize (as _FP4Group) and the narrow
    projections [x W_b^T | x W_a^T | x A_i^T] from one pass over x (as _XProjections). Backward:
    dx = sum_i Q(dy_i) dgrad_i^T + dproj [W_b; W_a; A_i], the second term added by rb2_lora_up in
    one pass over the first (no [M, hidden] product of its own and no autograd add), and the LoRA
    down-projections' dA_i as _XProjections computes them."""

    @staticmethod
    def forward(ctx, x, stochastic, w_frozen, weights, *As):
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
            x2 = x2.contiguous()
        q = N.quantize_activation(x2, weights[0].use_rht)
        ys = tuple(N._gemm_to(q, w.fprop, x.dtype).reshape(*x.shape[:-1], w.out_features) for w in weights)
        W = torch.cat([w_frozen.to(torch.bfloat16)] + [a.to(torch.bfloat16) for a in As], 0).contiguous()
        proj = narrow_product(x2, W)
        ctx.save_for_backward(x2, W)
        ctx.weights, ctx.stochastic, ctx.xshape = weights, stochastic, x.shape
        ctx.n_frozen, ctx.ranks = w_frozen.shape[0], [a.shape[0] for a in As]
        return (*ys, proj.reshape(*x.shape[:-1], W.shape[0]))

    @staticmethod
    def backward(ctx, *grads):
        x2, W = ctx.saved_tensors
        dys, dproj = grads[:-1], grads[-1]
        need_dx = ctx.needs_input_grad[0]
        dx = None
        if need_dx:  # as the reference, no NVFP4 dgrad when x needs no gradient
            for w, dy in zip(ctx.weights, dys):
                if dy is None:
                    continue
                d = N.quantize_activation(dy.reshape(-1, w.out_features), w.use_rht, stochastic=ctx.stochastic)
                part = N._gemm_to(d, w.dgrad, dy.dtype)
                dx = part if dx is None else dx + part
        gA = [None] * len(ctx.ranks)
        if dproj is not None:
            d2 = dproj.reshape(-1, dproj.shape[-1]).to(torch.bfloat16)
            off = ctx.n_frozen
            need = [ctx.needs_input_grad[4 + i] for i in range(len(ctx.ranks))]
            dh_all = d2[:, off:off + sum(ctx.ranks)]
            if any(need):
                if LORA_WGRAD and _wgrad_ok(x2, dh_all):
                    dA = lora_wgrad(x2, dh_all, 1.0, transposed=True)
                    o = 0
                    for i, r in enumerate(ctx.ranks):
                        gA[i] = dA[o:o + r] if need[i] else None
                        o += r
                else:
                    for i, r in enumerate(ctx.ranks):
                        gA[i] = (d2[:, off:off + r].t() @ x2).float() if need[i] else None
                        off += r
            if need_dx:
                wt = W.t().contiguous()  # [hidden, n]: the narrow weights as the up-projection's B
                if dx is not None and _use_up(dx, d2, wt):
                    dx = lora_up(dx, d2, wt, 1.0, 1)
                else:
                    dx = d2 @ W if dx is None else dx + d2 @ W
        return (None if dx is None else dx.reshape(ctx.xshape), None, None, None, *gA)


# The block's input projections as one function (_InProj) when both in_proj_qkv and in_proj_z are
# NVFP4; off, _FP4Group and _XProjections with autograd summing their input gradients.
FUSED_IN_PROJ = True


class _ConvSiLU(torch.autograd.Function):
    """Returns the conv output split into contiguous [B, T, s1], [B, T, s2 - s1], [B, T, C - s2]
    tensors (q, k, v of the block) written directly by the kernel, and (with ``want_state``) the
    next call's prefix [B, C, 3]. ``prev`` is the cached prefix (None = zeros); it gets no gradient."""

    @staticmethod
    def forward(ctx, x, w, s1, s2, prev, want_state, state_out):
        B, T, C = x.shape
        x = x.contiguous()
        w4 = w.reshape(C, 4).to(torch.bfloat16).contiguous()
        if prev is not None:
            prev = prev.to(device=x.device, dtype=torch.bfloat16).contiguous()
            if prev.shape != (B, C, 3):
                raise ValueError(f"recant_b200.conv_silu: conv state must be [{B}, {C}, 3], got {tuple(prev.shape)}")
        outs = [torch.empty(B, T, n, dtype=torch.bfloat16, device=x.device) for n in (s1, s2 - s1, C - s2)]
        if state_out is not None:
            if state_out.shape != (B, C, 3) or state_out.dtype != torch.bfloat16 or not state_out.is_contiguous():
                raise ValueError(f"recant_b200.conv_silu: state_out must be a contiguous bf16 [{B}, {C}, 3] tensor")
            state = state_out
        else:
            state = torch.empty(B, C, 3, dtype=torch.bfloat16, device=x.device) if want_state else None
        L.check(L.lib().rb2_conv_silu_fwd(_p(x), _p(w4), _p(prev), B, T, C, 4, *[_p(o) for o in outs], s1, s2,
                                          _p(state), _stream(x.device)), "conv_silu_fwd")
        ctx.save_for_backward(x, w4, prev)
        ctx.s1, ctx.s2 = s1, s2
        if state is not None:
            ctx.mark_non_differentiable(state)
        return (*outs, state)

    @staticmethod
    def backward(ctx, *grads):
        x, w4, prev = ctx.saved_tensors
        B, T, C = x.shape
        widths = (ctx.s1, ctx.s2 - ctx.s1, C - ctx.s2)
        dys = [torch.zeros(B, T, n, dtype=torch.bfloat16, device=x.device) if d is None
               else d.to(torch.bfloat16).contiguous() for d, n in zip(grads[:3], widths)]
        dx = torch.empty_like(x)
        L.check(L.lib().rb2_conv_silu_bwd(_p(x), _p(w4), _p(prev), *[_p(d) for d in dys], ctx.s1, ctx.s2, B, T, C, 4,
                                          _p(dx), _stream(x.device)), "conv_silu_bwd")
        return dx, None, None, None, None, None, None


class _Gates(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, A_log, dt_bias):
        H = a.shape[-1]
        a, b = a.to(torch.bfloat16).contiguous(), b.to(torch.bfloat16).contiguous()
        al, db_ = A_log.float().contiguous(), dt_bias.float().contiguous()
        g = torch.empty(a.shape, dtype=torch.float32, device=a.device)
        beta = torch.empty_like(b)
        L.check(L.lib().rb2_gdn_gates_fwd(_p(a), _p(b), _p(al), _p(db_), a.numel(), H, _p(g), _p(beta),
                                          _stream(a.device)), "gdn_gates_fwd")
        ctx.save_for_backward(a, beta, al, db_)
        return g, beta

    @staticmethod
    def backward(ctx, dg, dbeta):
        a, beta, al, db_ = ctx.saved_tensors
        H = a.shape[-1]
        dg = torch.zeros_like(a, dtype=torch.float32) if dg is None else dg.float().contiguous()
        dbeta = torch.zeros_like(beta) if dbeta is None else dbeta.to(torch.bfloat16).contiguous()
        da, db = torch.empty_like(a), torch.empty_like(beta)
        L.check(L.lib().rb2_gdn_gates_bwd(_p(a), _p(beta), _p(al), _p(db_), _p(dg), _p(dbeta), a.numel(), H, _p(da),
                                          _p(db), _stream(a.device)), "gdn_gates_bwd")
        return da, db, None, None


class _GatedRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, z, w, eps):
        x, z = x.to(torch.bfloat16).contiguous(), z.to(torch.bfloat16).contiguous()
        wf = w.float().contiguous()
        rows = x.numel() // 128
        y = torch.empty_like(x)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        L.check(L.lib().rb2_gated_rmsnorm_fwd(_p(x), _p(z), _p(wf), rows, 128, float(eps), _p(y), _p(rstd),
                                              _stream(x.device)), "gated_rmsnorm_fwd")
        ctx.save_for_backward(x, z, wf, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, z, wf, rstd = ctx.saved_tensors
        dy = dy.to(torch.bfloat16).contiguous()
        dx, dz = torch.empty_like(x), torch.empty_like(z)
        L.check(L.lib().rb2_gated_rmsnorm_bwd(_p(x), _p(z), _p(wf), _p(rstd), _p(dy), x.numel() // 128, 128, _p(dx),
                                              _p(dz), _stream(x.device)), "gated_rmsnorm_bwd")
        return dx, dz, None, None


class _GatedRMSNormQuant(torch.autograd.Function):
    """The gated RMSNorm whose output feeds an NVFP4 projection, fused with that projection's
    activation quantize (rb2_gated_rmsnorm_nvfp4_fwd): returns y and the NVFP4 codes, scales,
    blocked scales and global scale of quantize(rht(y)) for y viewed as [M, K] (RN, as
    quantize_activation in the forward, nvfp4.py:144-149). The quantized parts get no gradient;
    y's backward is the gated norm's."""

    @staticmethod
    def forward(ctx, x, z, w, eps, K, use_rht):
        x, z = x.to(torch.bfloat16).contiguous(), z.to(torch.bfloat16).contiguous()
        wf = w.float().contiguous()
        rows = x.numel() // 128
        M = rows * 128 // K
        y = torch.empty_like(x)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        codes = torch.empty(M, K // 2, dtype=torch.uint8, device=x.device)
        scales = torch.empty(M, K // 16, dtype=torch.uint8, device=x.device)
        blocked = torch.empty(N.blocked_size(M, K // 16), dtype=torch.uint8, device=x.device)
        gscale = torch.empty((), dtype=torch.float32, device=x.device)
        lib = L.lib()
        wsb = lib.rb2_nvfp4_quantize_workspace_size(M, K)
        ws = torch.empty(wsb, dtype=torch.uint8, device=x.device)
        L.check(lib.rb2_gated_rmsnorm_nvfp4_fwd(_p(x), _p(z), _p(wf), rows, 128, float(eps), _p(y), _p(rstd), M, K,
                                                int(use_rht), _p(codes), _p(scales), _p(blocked), _p(gscale), _p(ws),
                                                wsb, _stream(x.device)), "gated_rmsnorm_nvfp4_fwd")
        ctx.save_for_backward(x, z, wf, rstd)
        ctx.mark_non_differentiable(codes, scales, blocked, gscale)
        return y, codes, scales, blocked, gscale

    @staticmethod
    def backward(ctx, dy, *unused):
        dx, dz, _, _ = _GatedRMSNorm.backward(ctx, dy)
        return dx, dz, None, None, None, None


def gated_rmsnorm_quant(x, z, weight, K, use_rht=True, eps=1e-6):
    """RMSNormGated over rows of 128 and the NVFP4 quantize of its output viewed as [M, K]:
    (y, FP4Tensor) -- what ``out_proj(gated_rmsnorm(...))`` computes in two passes."""
    y, codes, scales, blocked, gscale = _GatedRMSNormQuant.apply(x, z, weight, eps, K, use_rht)
    M = codes.shape[0]
    return y, N.FP4Tensor(codes, scales.view(torch.float8_e4m3fn), gscale, (M, K), blocked)


def conv_silu(x, weight, s1, s2, prev=None, want_state=False, state_out=None):
    """silu(causal depthwise conv1d(x, weight [C, 1, 4])), x [B, T, C] bf16 (layers.py:157-168), split
    into channels [0, s1), [s1, s2), [s2, C) as three contiguous tensors (layers.py:169). ``prev``:
    the cached prefix [B, C, 3] (None = zeros). With ``want_state`` a fourth result is the next
    prefix, the last 3 tokens of cat(prev, x) (layers.py:165-166), written to ``state_out`` when
    given (which may be ``prev`` itself: updated in place); otherwise it is None."""
    q, k, v, state = _ConvSiLU.apply(x, weight, s1, s2, prev, want_state, state_out)
    return (q, k, v, state) if want_state else (q, k, v)


def gdn_gates(a, b, A_log, dt_bias):
    """(g, beta) = (-exp(A_log) softplus(a + dt_bias) fp32, sigmoid(b))  (fused_ops.py:32-33, layers.py:154)."""
    return _Gates.apply(a, b, A_log, dt_bias)


def gated_rmsnorm(x, z, weight, eps=1e-6):
    """RMSNormGated over rows of 128 (fused_ops.py:11-16, layers.py:23-34)."""
    return _GatedRMSNorm.apply(x, z, weight, eps)


class _FP4Group(torch.autograd.Function):
    """y_i = x . W_i^T for NVFP4 weights sharing one quantization of x (RN); backward: dx = sum_i
    Q(rht(dy_i)) . dgrad_i^T with stochastic rounding, as FP4Linear (nvfp4.py:151-170)."""

    @staticmethod
    def forward(ctx, x, stochastic, a_pre, *weights):
        x2 = x.reshape(-1, weights[0].in_features)
        # a_pre: x already quantized by its producer (gated_rmsnorm_quant), else quantized here
        a = N.quantize_activation(x2, weights[0].use_rht) if a_pre is None else a_pre
        ys = tuple(N._gemm_to(a, w.fprop, x.dtype).reshape(*x.shape[:-1], w.out_features) for w in weights)
        ctx.weights, ctx.stochastic, ctx.xshape = weights, stochastic, x.shape
        return ys

    @staticmethod
    def backward(ctx, *dys):
        dx = None
        for w, dy in zip(ctx.weights, dys):
            if dy is None:
                continue
            d = N.quantize_activation(dy.reshape(-1, w.out_features), w.use_rht, stochastic=ctx.stochastic)
            part = N._gemm_to(d, w.dgrad, dy.dtype)
            dx = part if dx is None else dx + part
        return (None if dx is None else dx.reshape(ctx.xshape), None, None, *([None] * len(ctx.weights)))


class _FP4LoRAGroup(torch.autograd.Function):
    """NVFP4 linears with LoRA sharing one input x: the activation is quantized once, h = x cat(A_i)^T
    is one cuBLAS product, and each member's (alpha / r) h_i B_i^T is added inside its NVFP4 GEMM's
    epilogue, rounded as the reference's ops round it (``mode`` 0: grouped_linear's one addmm per
    member, layers.py:86-97; 1: QLinear.forward's three ops, layers.py:65-70). Backward:
    the NVFP4 dgrads as _FP4Group, and the LoRA products dB_i = s dy_i^T h_i, dh_i = s dy_i B_i,
    dA = dh^T x, dx += dh cat(A_i) through cuBLAS."""

    @staticmethod
    def forward(ctx, x, stochastic, mode, weights, scales, *ab):
        k = weights[0].in_features
        x2 = x.reshape(-1, k)
        dt = x.dtype
        A = [t.to(dt) for t in ab[0::2]]
        B = [t.to(dt).contiguous() for t in ab[1::2]]
        a = N.quantize_activation(x2, weights[0].use_rht)
        h = x2 @ torch.cat(A, 0).t()
        ys, off = [], 0
        for w, b, sc in zip(weights, B, scales):
            r = b.shape[1]
            y = N.gemm_b200(a, w.fprop, out_dtype=dt, lora=(h[:, off:off + r], b, sc), lora_mode=mode)
            ys.append(y.reshape(*x.shape[:-1], w.out_features))
            off += r
        ctx.save_for_backward(x2, h, *A, *B)
        ctx.weights, ctx.scales, ctx.stochastic, ctx.xshape = weights, scales, stochastic, x.shape
        ctx.n = len(weights)
        return tuple(ys)

    @staticmethod
    def backward(ctx, *dys):
        x2, h, *ab = ctx.saved_tensors
        A, B = ab[:ctx.n], ab[ctx.n:]
        need_dx = ctx.needs_input_grad[0]  # as the reference, no NVFP4 dgrad when x needs no gradient
        dx, dhs, dBs, off = None, [], [], 0
        for w, b, sc, dy in zip(ctx.weights, B, ctx.scales, dys):
            r = b.shape[1]
            hi = h[:, off:off + r]
            off += r
            if dy is None:
                dhs.append(torch.zeros_like(hi))
                dBs.append(torch.zeros(b.shape, dtype=torch.float32, device=b.device))
                continue
            d2 = dy.reshape(-1, w.out_features).to(x2.dtype)
            if need_dx:
                q = N.quantize_activation(d2, w.use_rht, stochastic=ctx.stochastic)
                part = N._gemm_to(q, w.dgrad, d2.dtype)
                dx = part if dx is None else dx + part
            dBs.append((d2.t() @ hi).float() * sc)
            dhs.append((d2 @ b) * sc)
        dh = torch.cat(dhs, 1)
        dA = (dh.t() @ x2).float()
        if need_dx:
            dxl = dh @ torch.cat(A, 0)
            dx = dxl if dx is None else dx + dxl
        grads, off = [], 0
        for a_, b_, db in zip(A, B, dBs):
            r = a_.shape[0]
            grads += [dA[off:off + r], db]
            off += r
        return (None if dx is None else dx.reshape(ctx.xshape), None, None, None, None, *grads)


class _LoRAAddmm(torch.autograd.Function):
    """grouped_linear's LoRA up-projection, one addmm per member as the reference's (layers.py:86-97):
    y2 + s h2 B^T with B the fp32 factor cast to bf16, on rb2_lora_up (mode 0: addmm's rounding);
    backward as addmm's autograd (dy to y2, dh = (dy B) s in bf16) with dB from rb2_lora_wgrad."""

    @staticmethod
    def forward(ctx, y2, h2, B, s):
        b = B.to(y2.dtype)
        ctx.save_for_backward(h2, b)
        ctx.s = s
        if _use_up(y2, h2, b):
            return lora_up(y2, h2, b, s, 0)
        return torch.addmm(y2, h2, b.t(), alpha=s)

    @staticmethod
    def backward(ctx, dout):
        h2, b = ctx.saved_tensors
        s = ctx.s
        dh = _alpha(dout @ b, s) if ctx.needs_input_grad[1] else None
        dB = None
        if ctx.needs_input_grad[2]:
            dB = lora_wgrad(dout, h2, s) if LORA_WGRAD and _wgrad_ok(dout, h2) else _alpha(h2.t() @ dout, s).t().float()
        return (dout if ctx.needs_input_grad[0] else None), dh, dB, None


class _LoRAQLinear(torch.autograd.Function):
    """QLinear.forward's LoRA term as the reference's three bf16 ops (layers.py:65-70): h = x2 A^T,
    y2 + (h B^T) s, with A, B the fp32 factors cast to bf16; the up-projection and the add in one
    pass on rb2_lora_up (mode 1: the three ops' roundings). Backward as their autograd, with dA and
    dB from rb2_lora_wgrad."""

    @staticmethod
    def forward(ctx, x2, y2, A, B, s):
        a, b = A.to(x2.dtype), B.to(x2.dtype)
        h = x2 @ a.t()
        ctx.save_for_backward(x2, h, a, b)
        ctx.s = s
        if _use_up(y2, h, b):
            return lora_up(y2, h, b, s, 1)
        return y2 + (h @ b.t()) * s

    @staticmethod
    def backward(ctx, dout):
        x2, h, a, b = ctx.saved_tensors
        s = ctx.s
        # the gradient of (h B^T) is dt = dout * s in bf16; when s is a power of two that scaling is
        # exact and commutes with every rounding below, so it is applied to the products instead of
        # materialising dt (the same values, one pass over [M, N] fewer)
        fold = LORA_WGRAD and _pow2(s) and _wgrad_ok(dout, h)
        dt = None if fold else dout * s
        dB = None
        if ctx.needs_input_grad[3]:
            if fold:
                dB = lora_wgrad(dout, h, s)
            else:
                dB = lora_wgrad(dt, h, 1.0) if LORA_WGRAD and _wgrad_ok(dt, h) else (h.t() @ dt).t().float()
        dx = dA = None
        if ctx.needs_input_grad[0] or ctx.needs_input_grad[2]:
            dh = (dout @ b) * s if fold else dt @ b
            if ctx.needs_input_grad[2]:
                dA = (lora_wgrad(x2, dh, 1.0, transposed=True) if LORA_WGRAD and _wgrad_ok(x2, dh)
                      else (x2.t() @ dh).t().float())
            if ctx.needs_input_grad[0]:
                dx = dh @ a
        return dx, (dout if ctx.needs_input_grad[1] else None), dA, dB, None


class _FP4QLinear(torch.autograd.Function):
    """QLinear.forward with an NVFP4 base and LoRA (layers.py:62-70) as one function: y = Q(x) W^T
    (the activation quantized once, or given as ``a_pre``), then y + (h B^T) s on rb2_lora_up with
    h = x A^T, rounded as the reference's three ops. Backward: the NVFP4 dgrad as FP4Linear's
    (nvfp4.py:151-170) and the LoRA gradients as _LoRAQLinear's; x's two gradient contributions are
    summed inside rb2_lora_up (dx = bf16(dx_base + bf16(dh A)), the sum autograd would form from
    the two ops) instead of materialising dh A and adding it in another pass."""

    @staticmethod
    def forward(ctx, x2, stochastic, a_pre, w, A, B, s):
        a, b = A.to(x2.dtype), B.to(x2.dtype)
        q = N.quantize_activation(x2, w.use_rht) if a_pre is None else a_pre
        y = N._gemm_to(q, w.fprop, x2.dtype).to(x2.dtype)
        h = x2 @ a.t()
        ctx.save_for_backward(x2, h, a, b)
        ctx.s, ctx.w, ctx.stochastic = s, w, stochastic
        return lora_up(y, h, b, s, 1) if _use_up(y, h, b) else y + (h @ b.t()) * s

    @staticmethod
    def backward(ctx, dout):
        x2, h, a, b = ctx.saved_tensors
        s, w = ctx.s, ctx.w
        fold = LORA_WGRAD and _pow2(s) and _wgrad_ok(dout, h)
        dt = None if fold else dout * s
        dB = None
        if ctx.needs_input_grad[5]:
            if fold:
                dB = lora_wgrad(dout, h, s)
            else:
                dB = lora_wgrad(dt, h, 1.0) if LORA_WGRAD and _wgrad_ok(dt, h) else (h.t() @ dt).t().float()
        dx = dA = None
        if ctx.needs_input_grad[0] or ctx.needs_input_grad[4]:
            dh = (dout @ b) * s if fold else dt @ b
            if ctx.needs_input_grad[4]:
                dA = (lora_wgrad(x2, dh, 1.0, transposed=True) if LORA_WGRAD and _wgrad_ok(x2, dh)
                      else (x2.t() @ dh).t().float())
            if ctx.needs_input_grad[0]:
                d = N.quantize_activation(dout, w.use_rht, stochastic=ctx.stochastic)
                dx_base = N._gemm_to(d, w.dgrad, dout.dtype).to(dout.dtype)
                at = a.t().contiguous()  # [in, r]: A's rows as the up-projection's B operand
                dx = lora_up(dx_base, dh, at, 1.0, 1) if _use_up(dx_base, dh, at) else dx_base + dh @ a
        return dx, None, None, None, dA, dB, None


def _alpha(t, s):
    """torch's maybe_multiply: the product times alpha unless alpha is 1."""
    return t if s == 1 else t * s


def _lora_kernels_ok(x):
    return (LORA_WGRAD or LORA_UP) and x.is_cuda and x.dtype == torch.bfloat16


# Add LoRA inside the NVFP4 GEMM epilogue (_FP4LoRAGroup) instead of the reference's addmm through
# cuBLAS. Off by default: measured at config 2 it is slower (5.75 vs 5.40 ms per block step; the 16
# FMAs per output element on CUDA cores are not hidden behind the next tile), as is the decode step.
FUSED_LORA_EPILOGUE = False


def _fused_lora_ok(lins):
    return FUSED_LORA_EPILOGUE and all(l.fp4 is not None and l.lora_A is not None and l.lora_A.shape[0] in (8, 16) for l in lins) and \
        len({l.fp4.use_rht for l in lins}) == 1


class QLinear(nn.Module):
    """layers.py:36-70: NVFP4 base when quantizable (in, out % 16 == 0 and out >= 256), else a bf16
    dense weight; optional LoRA y += (alpha / r) (x A^T) B^T with fp32 A [r, in], B [out, r]."""

    def __init__(self, in_f, out_f):
        super().__init__()
        self.in_features, self.out_features = in_f, out_f
        self.weight = None          # bf16 dense weight when not quantized
        self.fp4 = None
        self.lora_A = self.lora_B = None
        self.lora_scale = 1.0
        self.stochastic_backward = True

    @property
    def quantizable(self):
        return self.in_features % 16 == 0 and self.out_features % 16 == 0 and self.out_features >= 256

    def load_weight(self, w, use_rht=True):
        if self.quantizable:
            self.fp4 = N.quantize_weight(w.detach(), use_rht)
            self.weight = None
        else:
            self.weight = w.detach().to(torch.bfloat16).contiguous()

    def add_lora(self, r, alpha, device):
        self.lora_A = nn.Parameter(torch.empty(r, self.in_features, device=device, dtype=torch.float32))
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self.lora_B = nn.Parameter(torch.zeros(self.out_features, r, device=device, dtype=torch.float32))
        self.lora_scale = alpha / r

    def lora(self, x, y, grouped=False):
        """y + (alpha / r) (x A^T) B^T: three bf16 ops as QLinear.forward (layers.py:65-70), or one
        addmm as grouped_linear's default path (layers.py:86-97)."""
        if self.lora_A is None:
            return y
        if not grouped and _lora_kernels_ok(x) and y.shape == x.shape[:-1] + (self.out_features,):
            x2 = x.reshape(-1, self.in_features)
            o = _LoRAQLinear.apply(x2, y.reshape(-1, self.out_features), self.lora_A, self.lora_B, self.lora_scale)
            return o.reshape(*y.shape)
        h = x @ self.lora_A.to(x.dtype).t()
        if grouped:
            o = torch.addmm(y.reshape(-1, y.shape[-1]), h.reshape(-1, h.shape[-1]), self.lora_B.to(x.dtype).t(),
                            alpha=self.lora_scale)
            return o.reshape(*y.shape)
        return y + (h @ self.lora_B.to(x.dtype).t()) * self.lora_scale

    def forward(self, x, a_pre=None):
        """``a_pre``: x already quantized (the FP4Tensor of x, RN, with this weight's RHT setting),
        as the fused gated norm produces it; used by the NVFP4 base only."""
        if (self.fp4 is not None and self.lora_A is not None and LORA_UP and not _fused_lora_ok([self])
                and x.is_cuda and x.dtype == torch.bfloat16 and self.lora_A.shape[0] <= 64):
            x2 = x.reshape(-1, self.in_features)
            y = _FP4QLinear.apply(x2, self.stochastic_backward, a_pre, self.fp4, self.lora_A, self.lora_B,
                                  self.lora_scale)
            return y.reshape(*x.shape[:-1], self.out_features)
        if _fused_lora_ok([self]):
            (y,) = _FP4LoRAGroup.apply(x, self.stochastic_backward, 1, (self.fp4,), (self.lora_scale,),
                                       self.lora_A, self.lora_B)
            return y
        if self.fp4 is not None:
            (y,) = _FP4Group.apply(x, self.stochastic_backward, a_pre, self.fp4)
        else:
            y = x @ self.weight.t()
        return self.lora(x, y)


def grouped_linear(x, lins, h=None, base=None):
    """layers.py:72-97 with the activation quantized once for all NVFP4 members; the LoRA
    down-projections of all members come from one GEMM over x (x . cat(A_i)^T, as the reference's
    default path, layers.py:86-88), or are given as ``h`` (the members' x A_i^T side by side, e.g.
    from :class:`_XProjections`); each member's up-projection is one addmm as the reference's, or,
    with the fused LoRA epilogue switched on, is added inside its NVFP4 GEMM (ranks 8 and 16).
    ``base``: the NVFP4 members' products of x, in order, when already computed."""
    if _fused_lora_ok(lins):
        ab = [t for l in lins for t in (l.lora_A, l.lora_B)]
        return list(_FP4LoRAGroup.apply(x, lins[0].stochastic_backward, 0, tuple(l.fp4 for l in lins),
                                        tuple(l.lora_scale for l in lins), *ab))
    fp4 = [l for l in lins if l.fp4 is not None]
    outs = {}
    if base is not None:  # the NVFP4 products, already computed (by _InProj)
        outs = {id(l): y for l, y in zip(fp4, base)}
    elif fp4:
        ys = _FP4Group.apply(x, fp4[0].stochastic_backward, None, *[l.fp4 for l in fp4])
        outs = {id(l): y for l, y in zip(fp4, ys)}
    base = [outs[id(l)] if id(l) in outs else x @ l.weight.t() for l in lins]
    act = [l for l in lins if l.lora_A is not None]
    if not act:
        return base
    if h is None:
        h = x @ torch.cat([l.lora_A for l in act], 0).to(x.dtype).t()
    res, off = [], 0
    for l, y in zip(lins, base):
        if l.lora_A is None:
            res.append(y)
            continue
        r = l.lora_A.shape[0]
        hi = h[..., off:off + r].reshape(-1, r)
        off += r
        if _lora_kernels_ok(x):
            o = _LoRAAddmm.apply(y.reshape(-1, l.out_features), hi, l.lora_B, l.lora_scale)
        else:
            o = torch.addmm(y.reshape(-1, l.out_features), hi, l.lora_B.to(x.dtype).t(), alpha=l.lora_scale)
        res.append(o.reshape(*y.shape))
    return res


class GDNBlock(nn.Module):
    """``GatedDeltaNet`` (layers.py:133-182) on B200. Parameters keep the reference's names;
    :meth:`from_reference` copies a reference block's weights (and LoRA) into it."""

    def __init__(self, hidden, Hk, Hv, d=128, conv_k=4, eps=1e-6):
        super().__init__()
        if d != 128 or conv_k != 4:
            raise ValueError("recant_b200.GDNBlock: head dim 128 and conv kernel 4 only")
        self.hidden, self.Hk, self.Hv, self.d, self.eps = hidden, Hk, Hv, d, eps
        self.key_dim, self.value_dim = Hk * d, Hv * d
        self.conv_dim = 2 * self.key_dim + self.value_dim
        self.in_proj_qkv = QLinear(hidden, self.conv_dim)
        self.in_proj_z = QLinear(hidden, self.value_dim)
        self.in_proj_b = QLinear(hidden, Hv)
        self.in_proj_a = QLinear(hidden, Hv)
        self.out_proj = QLinear(self.value_dim, hidden)
        self.register_buffer("conv_weight", torch.zeros(self.conv_dim, 1, conv_k, dtype=torch.bfloat16))
        self.register_buffer("dt_bias", torch.ones(Hv))
        self.register_buffer("A_log", torch.zeros(Hv))
        self.register_buffer("norm_weight", torch.ones(d))

    def projections(self):
        return [self.in_proj_qkv, self.in_proj_z, self.in_proj_b, self.in_proj_a, self.out_proj]

    def set_stochastic_backward(self, on: bool):
        for l in self.projections():
            l.stochastic_backward = on

    @classmethod
    def from_reference(cls, ref, device="cuda"):
        """Build from a reference ``GatedDeltaNet`` (unquantized weights, optional LoRA)."""
        c = ref.c
        blk = cls(c.hidden_size, c.linear_num_key_heads, c.linear_num_value_heads, c.linear_value_head_dim,
                  c.linear_conv_kernel_dim, c.rms_norm_eps).to(device)
        for name in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj"):
            src, dst = getattr(ref, name), getattr(blk, name)
            if src.weight is None:
                raise ValueError("from_reference needs the reference block's unquantized weights")
            dst.load_weight(src.weight.data.to(device))
            if src.lora_A is not None:
                dst.lora_A = nn.Parameter(src.lora_A.detach().float().to(device).clone())
                dst.lora_B = nn.Parameter(src.lora_B.detach().float().to(device).clone())
                dst.lora_scale = src.lora_scale
        blk.conv_weight.copy_(ref.conv1d.weight.detach().to(device, torch.bfloat16))
        blk.dt_bias.copy_(ref.dt_bias.detach().float())
        blk.A_log.copy_(ref.A_log.detach().float())
        blk.norm_weight.copy_(ref.norm.weight.detach().float())
        return blk

    @classmethod
    def from_state(cls, sd, hidden, Hk, Hv, lora_scale=2.0, device="cuda"):
        """Build from reference-named tensors: ``<proj>.weight`` (unquantized), optional
        ``<proj>.lora_A`` / ``.lora_B``, ``conv1d.weight``, ``dt_bias``, ``A_log``, ``norm.weight``."""
        blk = cls(hidden, Hk, Hv).to(device)
        for name in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj"):
            dst = getattr(blk, name)
            dst.load_weight(sd[name + ".weight"].to(device, torch.bfloat16))
            if name + ".lora_A" in sd:
                dst.lora_A = nn.Parameter(sd[name + ".lora_A"].float().to(device).clone())
                dst.lora_B = nn.Parameter(sd[name + ".lora_B"].float().to(device).clone())
                dst.lora_scale = lora_scale
        blk.conv_weight.copy_(sd["conv1d.weight"].to(device, torch.bfloat16))
        blk.dt_bias.copy_(sd["dt_bias"].to(device, torch.bfloat16).float())
        blk.A_log.copy_(sd["A_log"].to(device, torch.bfloat16).float())
        blk.norm_weight.copy_(sd["norm.weight"].to(device, torch.bfloat16).float())
        return blk

    def forward(self, x, cache=None, pos_offset=0, inplace_cache=False):
        """x [B, T, hidden] -> [B, T, hidden]. ``cache``: any object with ``conv_state`` ([B, C, 3]
        bf16 or None) and ``rec_state`` ([B, Hv, 128, 128] fp32 or None) attributes -- the
        reference's ``LayerCache`` (layers.py:111-130) or :class:`LayerCache` here; both are read
        and replaced as GatedDeltaNet.forward does (layers.py:158-166, 177-180). With
        ``inplace_cache`` (a short call without gradient, both states present) the states are
        updated in their own storage instead, so their addresses stay fixed (what a captured CUDA
        graph needs). ``pos_offset`` is accepted for the reference's signature and unused."""
        B, T, _ = x.shape
        d = self.d
        ins = [self.in_proj_qkv, self.in_proj_z]
        lora_ins = [l for l in ins if l.lora_A is not None]
        dense_ba = self.in_proj_b.weight is not None and self.in_proj_a.weight is not None
        if (dense_ba and not _fused_lora_ok(ins)
                and _narrow_ok(x, 2 * self.Hv + sum(l.lora_A.shape[0] for l in lora_ins))):
            # one pass over x: b, a and the LoRA down-projections of in_proj_qkv / in_proj_z
            wba = torch.cat([self.in_proj_b.weight, self.in_proj_a.weight], 0)
            base = None
            if FUSED_IN_PROJ and LORA_UP and all(l.fp4 is not None for l in ins):
                *base, proj = _InProj.apply(x, ins[0].stochastic_backward, wba, tuple(l.fp4 for l in ins),
                                            *[l.lora_A for l in lora_ins])
            else:
                proj = _XProjections.apply(x, wba, *[l.lora_A for l in lora_ins])
            b_lin, a = proj[..., :self.Hv], proj[..., self.Hv:2 * self.Hv]
            qkv, z = grouped_linear(x, ins, h=proj[..., 2 * self.Hv:] if lora_ins else None, base=base)
        else:
            qkv, z = grouped_linear(x, ins)
            if dense_ba:  # one N = 2 Hv GEMM
                ba = x @ torch.cat([self.in_proj_b.weight, self.in_proj_a.weight], 0).t()
                b_lin, a = ba[..., :self.Hv], ba[..., self.Hv:]
            else:
                b_lin, a = self.in_proj_b(x), self.in_proj_a(x)
        inplace = (inplace_cache and cache is not None and cache.conv_state is not None
                   and cache.rec_state is not None and T <= RECURRENT_MAX_T and not torch.is_grad_enabled())
        if cache is None:
            q, k, v = conv_silu(qkv, self.conv_weight, self.key_dim, 2 * self.key_dim)
        else:
            q, k, v, state = conv_silu(qkv, self.conv_weight, self.key_dim, 2 * self.key_dim,
                                       prev=cache.conv_state, want_state=True,
                                       state_out=cache.conv_state if inplace else None)
            if not inplace:  # in place, the cache keeps its own tensor (state aliases it)
                cache.conv_state = state
        q = q.view(B, T, self.Hk, d)
        k = k.view(B, T, self.Hk, d)
        v = v.view(B, T, self.Hv, d)
        g, beta = gdn_gates(a, b_lin, self.A_log, self.dt_bias)
        if cache is None:
            core, _ = gdn_b200(q, k, v, g, beta)
        elif inplace:
            core, _ = gdn_recurrent(q, k, v, g, beta, cache.rec_state, True, final_state_out=cache.rec_state)
        else:
            core, rec = gdn_b200(q, k, v, g, beta, initial_state=cache.rec_state, output_final_state=True)
            cache.rec_state = rec.detach()
        op = self.out_proj
        if (FUSE_NORM_QUANT and op.fp4 is not None and not _fused_lora_ok([op]) and core.dtype == torch.bfloat16
                and core.numel() // 16 > NORM_QUANT_MIN_BLOCKS):
            # the norm's pass also reduces the quantizer's global amax; out_proj gets the codes
            y, a = gated_rmsnorm_quant(core.reshape(-1, d), z.reshape(-1, d), self.norm_weight, op.in_features,
                                       op.fp4.use_rht, self.eps)
            return op(y.reshape(B, T, -1), a_pre=a)
        y = gated_rmsnorm(core.reshape(-1, d), z.reshape(-1, d), self.norm_weight, self.eps)
        return op(y.reshape(B, T, -1))


@dataclass
class LayerCache:
    """Per-layer decode state with the reference's fields (layers.py:111-130): the conv prefix
    [B, conv_dim, 3] and the recurrent state [B, Hv, 128, 128] fp32 (None before the first call)."""
    conv_state: torch.Tensor | None = None
    rec_state: torch.Tensor | None = None

    def fork(self) -> "LayerCache":
        return LayerCache(None if self.conv_state is None else self.conv_state.clone(),
                          None if self.rec_state is None else self.rec_state.clone())


class DecodeGraph:
    """The decode step of a :class:`GDNBlock` captured once in a CUDA graph and replayed per token: a
    fixed batch of B sequences, one new token each, the cache's conv prefix and fp32 recurrent
    state held in static tensors and updated in place by the kernels. A step is one copy of the new
    token into the static input and one graph replay, where the reference's engine runs the block's
    Python and torch ops for every token (serve/engine.py:107-119 -> layers.py:148-182).

    ``cache`` (fields ``conv_state`` / ``rec_state``, None = zeros) is adopted: after construction
    its two fields are the static tensors, holding the same values as before."""

    def __init__(self, blk: GDNBlock, cache, B: int):
        dev = blk.conv_weight.device
        bf = torch.bfloat16
        conv = torch.zeros(B, blk.conv_dim, 3, dtype=bf, device=dev)
        rec = torch.zeros(B, blk.Hv, blk.d, blk.d, dtype=torch.float32, device=dev)
        if cache.conv_state is not None:
            conv.copy_(cache.conv_state)
        if cache.rec_state is not None:
            rec.copy_(cache.rec_state)
        cache.conv_state, cache.rec_state = conv, rec
        self.blk, self.cache = blk, cache
        self.x = torch.zeros(B, 1, blk.hidden, dtype=bf, device=dev)
        saved = (conv.clone(), rec.clone())
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.no_grad(), torch.cuda.stream(side):
            for _ in range(2):  # warm-up (allocations, one-time attributes) outside the capture
                blk(self.x, cache, inplace_cache=True)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.out = blk(self.x, cache, inplace_cache=True)
        if cache.conv_state.data_ptr() != conv.data_ptr() or cache.rec_state.data_ptr() != rec.data_ptr():
            raise RuntimeError("recant_b200.DecodeGraph: the block did not update the cache in place")
        conv.copy_(saved[0])  # the warm-up steps advanced the states
        rec.copy_(saved[1])

    def __call__(self, x_t: torch.Tensor) -> torch.Tensor:
        """x_t [B, 1, hidden] -> [B, 1, hidden] (a view of a static buffer, valid until the next call)."""
        self.x.copy_(x_t)
        self.graph.replay()
        return self.out
