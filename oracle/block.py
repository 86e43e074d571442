"""GDN block oracle on the CPU -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates ``recant.model.layers.GatedDeltaNet.forward`` (recant/model/layers.py:148-182) with torch
CPU ops, for a bf16 block:
  qkv, z   = grouped_linear over NVFP4 QLinears -- quantize(rht(x)) round-to-nearest, the emulated
             GEMM (dequantize both operands, matmul; nvfp4.py:108-110, 144-170) cast to the
             activation dtype -- plus LoRA as one addmm y + (alpha / r) (x A^T) B^T (the default
             fused path, layers.py:86-97)
  beta, a  = sigmoid(x Wb^T), x Wa^T (bf16 dense: N < 256 is never quantized, layers.py:47-48)
  conv     = silu(conv1d(cat(prefix, qkv^T), w, groups=C))^T             (layers.py:157-166)
             prefix = zeros, or a cache's conv_state, which then becomes cat[..., -3:]
  q, k, v  = split(conv); g = -exp(A_log) softplus(a + dt_bias)          (fused_ops.py:32-33)
  core     = gdn_torch(q, k, v, g, beta) with q, k repeated to Hv        (layers.py:174-178; oracle.gdn)
             (with a cache: initial_state = rec_state, which becomes the final state)
  out      = QLinear_out(rmsnorm_gated(core, z))                          (fused_ops.py:11-16)
The backward is autograd over this graph. The NVFP4 linear's backward quantizes dy with
round-to-nearest here, where the reference draws stochastic rounding from torch's RNG: the B200
block is compared with stochastic rounding switched off. NVFP4 arithmetic comes from oracle.nvfp4
(bit-exact quantizer) and its emulated GEMM, the same float32 torch matmul as the reference.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import gdn as OG
from . import nvfp4 as ON


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).numpy()


class _FP4Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, fprop, dgrad, n_out):
        k = x.shape[-1]
        x2 = x.reshape(-1, k)
        dt = "bf16" if x.dtype == torch.bfloat16 else "f32"
        a = ON.quantize_activation(_np(x2), dt) + ((x2.shape[0], k),)
        y = torch.from_numpy(ON.gemm_emulated(a, fprop)).to(x.dtype)
        ctx.dgrad, ctx.k, ctx.dt, ctx.xshape = dgrad, k, dt, x.shape
        return y.reshape(*x.shape[:-1], n_out)

    @staticmethod
    def backward(ctx, dy):
        n = dy.shape[-1]
        d2 = dy.reshape(-1, n)
        d = ON.quantize_activation(_np(d2), ctx.dt) + ((d2.shape[0], n),)
        dx = torch.from_numpy(ON.gemm_emulated(d, ctx.dgrad)).to(dy.dtype)
        return dx.reshape(ctx.xshape), None, None, None


def qlinear(x, p, grouped=False):
    """p: {"fp4": (fprop, dgrad) from oracle.nvfp4.quantize_weight | "weight": dense tensor,
    optional "A" [r, in], "B" [out, r] (fp32, requires_grad), "scale"}. LoRA as QLinear.forward
    (layers.py:65-70), or with ``grouped`` as grouped_linear's default path, one addmm per member
    (layers.py:86-97)."""
    if "fp4" in p:
        y = _FP4Linear.apply(x, p["fp4"][0], p["fp4"][1], p["n_out"])
    else:
        y = F.linear(x, p["weight"].to(x.dtype))
    if p.get("A") is not None:
        if grouped:
            h = F.linear(x, p["A"].to(x.dtype))
            o = torch.addmm(y.reshape(-1, y.shape[-1]), h.reshape(-1, h.shape[-1]), p["B"].to(x.dtype).t(),
                            alpha=p["scale"])
            y = o.reshape(*y.shape)
        else:
            y = y + F.linear(F.linear(x, p["A"].to(x.dtype)), p["B"].to(x.dtype)) * p["scale"]
    return y


def quantized(weight: torch.Tensor, lora=None) -> dict:
    """An NVFP4 QLinear from a (bf16) weight [out, in]; lora = (A, B, scale) or None."""
    fprop, dgrad = ON.quantize_weight(_np(weight))
    p = {"fp4": (fprop, dgrad), "n_out": weight.shape[0]}
    if lora is not None:
        p["A"], p["B"], p["scale"] = lora
    return p


def block_forward(x, P, Hk, Hv, d=128, eps=1e-6, cache=None):
    """x [B, T, hidden] bf16; P: {"in_proj_qkv", "in_proj_z", "out_proj": qlinear dicts,
    "in_proj_b", "in_proj_a": {"weight"}, "conv": [C, 1, 4], "A_log", "dt_bias": [Hv],
    "norm": [d]} -> [B, T, hidden]. ``cache``: an object with ``conv_state`` / ``rec_state`` (None
    at first), read and replaced as GatedDeltaNet.forward does with a LayerCache (layers.py:158-166,
    177-180)."""
    b, t, _ = x.shape
    key_dim, value_dim = Hk * d, Hv * d
    conv_dim = 2 * key_dim + value_dim
    qkv = qlinear(x, P["in_proj_qkv"], grouped=True)
    z = qlinear(x, P["in_proj_z"], grouped=True).reshape(b, t, -1, d)
    beta = qlinear(x, P["in_proj_b"]).sigmoid()
    a = qlinear(x, P["in_proj_a"])
    mixed = qkv.transpose(1, 2)
    prev = cache.conv_state if cache is not None else None
    prev = prev if prev is not None else torch.zeros(b, conv_dim, 3, dtype=mixed.dtype)
    cat = torch.cat([prev.to(mixed.dtype), mixed], dim=-1)
    conv = F.silu(F.conv1d(cat, P["conv"].to(mixed.dtype), groups=conv_dim)).transpose(1, 2)
    if cache is not None:
        cache.conv_state = cat[..., -3:].detach().clone()
    q, k, v = torch.split(conv, [key_dim, key_dim, value_dim], dim=-1)
    q = q.reshape(b, t, Hk, d)
    k = k.reshape(b, t, Hk, d)
    v = v.reshape(b, t, Hv, d)
    g = -P["A_log"].float().exp() * F.softplus(a.float() + P["dt_bias"].float())
    init = cache.rec_state if cache is not None else None
    core, state = OG.gdn(q, k, v, g, beta, initial_state=init, output_final_state=cache is not None)
    if cache is not None:
        cache.rec_state = state.detach()
    core = core.to(x.dtype)
    xf = core.reshape(-1, d).float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = P["norm"].to(x.dtype) * y.to(x.dtype)
    y = (y * F.silu(z.reshape(-1, d).float())).to(x.dtype)
    return qlinear(y.reshape(b, t, -1), P["out_proj"])
