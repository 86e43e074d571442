"""NVFP4 quantizer and block-scaled GEMM on B200, shaped like recant/model/nvfp4.py.

* :class:`FP4Tensor` has the reference's fields (codes u8 [M,K/2], scales float8_e4m3fn [M,K/16],
  gscale fp32 0-d, shape) plus ``blocked``: the same scales in the 128x4 blocked swizzle that
  the GEMM consumes (nvfp4._to_blocked, nvfp4.py:112-119), produced by the quantizer itself.
* :func:`quantize_fast` is the drop-in for ``fp4_kernels.quantize_fast(x, use_rht, stochastic)``
  (recant/model/fp4_kernels.py:452-467) behind ``nvfp4._fast['quantize']`` (nvfp4.py:139-149):
  bit-exact codes/scales/gscale for round-to-nearest; stochastic rounding is unbiased.
* :func:`gemm_b200` is the drop-in for a ``GEMM_BACKENDS`` entry (nvfp4.py:108-125):
  ``fn(a, b) -> fp32 [M, N] = a . b^T * gA * gB``.
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field

import torch

from . import _lib as L

BLOCK = 16
# Up to this many rows of A the GEMM runs as rb2_nvfp4_gemv (each row of B read once by one warp),
# as long as A, dequantized with padding (K + K/8 floats per row), fits the kernel's shared memory
GEMV_MAX_M = 4
GEMV_MAX_ELEMS = 50_000
# Frozen weights keep the scales the GEMM reads for its B operand (the blocked layout, built once at
# quantisation) instead of rebuilding them every call
CACHE_WEIGHT_IMAGES = True
_DT = {torch.float32: L.F32, torch.bfloat16: L.BF16}


@dataclass
class FP4Tensor:
    codes: torch.Tensor
    scales: torch.Tensor
    gscale: torch.Tensor
    shape: tuple
    blocked: torch.Tensor | None = field(default=None, repr=False)
    gemm_images: torch.Tensor | None = field(default=None, repr=False)  # B-operand scales as the GEMM reads them


def blocked_size(rows: int, cols: int) -> int:
    return -(-rows // 128) * -(-cols // 4) * 512


def quantize_fast(x: torch.Tensor, use_rht: bool = True, stochastic: bool = False, seed: int | None = None) -> FP4Tensor:
    if not x.is_cuda or x.dim() != 2 or x.shape[1] % BLOCK or x.dtype not in _DT:
        raise ValueError(f"recant_b200.quantize_fast: need a CUDA 2-D float32/bfloat16 tensor with K % 16 == 0, "
                         f"got {x.dtype} {tuple(x.shape)} on {x.device}")
    x = x.contiguous()
    m, k = x.shape
    g = k // BLOCK
    codes = torch.empty(m, k // 2, dtype=torch.uint8, device=x.device)
    scales = torch.empty(m, g, dtype=torch.uint8, device=x.device)
    blocked = torch.empty(blocked_size(m, g), dtype=torch.uint8, device=x.device)
    gscale = torch.empty((), dtype=torch.float32, device=x.device)
    lib = L.lib()
    wsb = lib.rb2_nvfp4_quantize_workspace_size(m, k)
    ws = torch.empty(wsb, dtype=torch.uint8, device=x.device)
    if stochastic and seed is None:
        seed = random.getrandbits(62)
    st = lib.rb2_nvfp4_quantize(L.ptr(x), m, k, _DT[x.dtype], int(use_rht), int(stochastic), int(seed or 0),
                                L.ptr(codes), L.ptr(scales), L.ptr(blocked), L.ptr(gscale), L.ptr(ws), wsb,
                                torch.cuda.current_stream(x.device).cuda_stream)
    L.check(st, "nvfp4_quantize")
    return FP4Tensor(codes, scales.view(torch.float8_e4m3fn), gscale, (m, k), blocked)


def blocked_scales(t) -> torch.Tensor:
    """The 128x4 blocked swizzle of an FP4 tensor's scales (computed on the GPU if absent)."""
    b = getattr(t, "blocked", None)
    if b is not None:
        return b
    rows, k = t.shape
    sc = t.scales.contiguous().view(torch.uint8)
    b = torch.empty(blocked_size(rows, k // BLOCK), dtype=torch.uint8, device=sc.device)
    L.check(L.lib().rb2_nvfp4_block_scales(L.ptr(sc), rows, k // BLOCK, L.ptr(b),
                                           torch.cuda.current_stream(sc.device).cuda_stream), "nvfp4_block_scales")
    return b


def gemm_images(t) -> torch.Tensor:
    """The scales the GEMM kernel reads for ``t`` as its B operand, kept on the tensor (frozen
    weights). The kernel reads the blocked layout in place, so these are the blocked scales."""
    if t.gemm_images is None:
        t.gemm_images = blocked_scales(t)
    return t.gemm_images


def gemm_b200(a, b, out_dtype=torch.float32, lora=None, lora_mode=0) -> torch.Tensor:
    """a . b^T * (gA gB) with a [M,K] and b [N,K] NVFP4 tensors; fp32 (or bf16) [M, N]. ``lora`` =
    (h [M, r] bf16, B [N, r] bf16, scale) adds scale * h B^T (QLinear's LoRA with h = x A^T,
    layers.py:65-70, 86-97), with bf16 output rounded as grouped_linear's addmm (``lora_mode`` 0)
    or as QLinear.forward's three ops (1)."""
    m, k = a.shape
    n, kb = b.shape
    if k != kb:
        raise ValueError(f"recant_b200.gemm_b200: K mismatch {k} vs {kb}")
    if not a.codes.is_cuda:
        raise ValueError("recant_b200.gemm_b200: operands must be CUDA tensors (no CPU path)")
    out = torch.empty(m, n, dtype=out_dtype, device=a.codes.device)
    lib = L.lib()
    if lora is None and 0 < m <= GEMV_MAX_M and n > 0 and k % 32 == 0 and m * (k + k // 8) <= GEMV_MAX_ELEMS:
        # a few rows of A (the decode step): read B once, one warp per row
        ga = a.gscale.reshape(1).to(torch.float32).contiguous()
        gb = b.gscale.reshape(1).to(torch.float32).contiguous()
        st = lib.rb2_nvfp4_gemv(L.ptr(a.codes.contiguous()), L.ptr(a.scales.contiguous().view(torch.uint8)), L.ptr(ga),
                                L.ptr(b.codes.contiguous()), L.ptr(b.scales.contiguous().view(torch.uint8)), L.ptr(gb),
                                m, n, k, L.ptr(out), _DT[out_dtype], torch.cuda.current_stream(a.codes.device).cuda_stream)
        L.check(st, "nvfp4_gemv")
        return out
    wsb = lib.rb2_nvfp4_gemm_workspace_size(m, n, k)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=a.codes.device)
    ga = a.gscale.reshape(1).to(torch.float32).contiguous()
    gb = b.gscale.reshape(1).to(torch.float32).contiguous()
    img = getattr(b, "gemm_images", None)
    h = bl = None
    r, ldh, sc = 0, 0, 0.0
    if lora is not None:
        h, bl, sc = lora
        if h.stride(-1) != 1 or h.dtype != torch.bfloat16 or h.shape[0] != m:
            raise ValueError("recant_b200.gemm_b200: LoRA h must be a bf16 [M, r] tensor with unit column stride")
        bl = bl.to(torch.bfloat16).contiguous()
        r, ldh = bl.shape[1], h.stride(0)
    st = lib.rb2_nvfp4_gemm_ex(L.ptr(a.codes.contiguous()), L.ptr(blocked_scales(a)), L.ptr(ga),
                               L.ptr(b.codes.contiguous()), L.ptr(blocked_scales(b)), L.ptr(gb), L.ptr(img),
                               L.ptr(h), ldh, L.ptr(bl), r, float(sc), int(lora_mode), m, n, k,
                               L.ptr(out), _DT[out_dtype], L.ptr(ws), wsb,
                               torch.cuda.current_stream(a.codes.device).cuda_stream)
    L.check(st, "nvfp4_gemm")
    L.check_status(ws, "nvfp4_gemm")
    return out


def gemm_pair_b200(a, b, out_dtype=torch.float32) -> torch.Tensor:
    """The product of :func:`gemm_b200` (no LoRA) on SM pairs: two-CTA clusters computing 256 x 256
    tiles (rb2_nvfp4_gemm_pair). Same results; slower than the one-SM kernel at the shapes measured,
    kept as the measured alternative."""
    m, k = a.shape
    n, kb = b.shape
    if k != kb:
        raise ValueError(f"recant_b200.gemm_pair_b200: K mismatch {k} vs {kb}")
    if not a.codes.is_cuda:
        raise ValueError("recant_b200.gemm_pair_b200: operands must be CUDA tensors (no CPU path)")
    out = torch.empty(m, n, dtype=out_dtype, device=a.codes.device)
    lib = L.lib()
    wsb = lib.rb2_nvfp4_gemm_workspace_size(m, n, k)
    ws = torch.empty(max(wsb, 1), dtype=torch.uint8, device=a.codes.device)
    ga = a.gscale.reshape(1).to(torch.float32).contiguous()
    gb = b.gscale.reshape(1).to(torch.float32).contiguous()
    st = lib.rb2_nvfp4_gemm_pair(L.ptr(a.codes.contiguous()), L.ptr(blocked_scales(a)), L.ptr(ga),
                                 L.ptr(b.codes.contiguous()), L.ptr(blocked_scales(b)), L.ptr(gb), m, n, k,
                                 L.ptr(out), _DT[out_dtype], L.ptr(ws), wsb,
                                 torch.cuda.current_stream(a.codes.device).cuda_stream)
    L.check(st, "nvfp4_gemm_pair")
    L.check_status(ws, "nvfp4_gemm_pair")
    return out


@dataclass
class FP4Weight:
    """Frozen NVFP4 weight with its fprop (Q(rht(W)) [N,K]) and dgrad (Q(rht(W^T)) [K,N]) copies,
    as recant/model/nvfp4.py:93-106."""
    fprop: FP4Tensor
    dgrad: FP4Tensor
    out_features: int
    in_features: int
    use_rht: bool


def quantize_weight(w: torch.Tensor, use_rht: bool = True) -> FP4Weight:
    """GPU quantize_weight (nvfp4.py:101-106): fp32 RHT, no re-rounding; bit-exact."""
    n, k = w.shape
    wf = w.detach().to(torch.float32).contiguous()
    fp = quantize_fast(wf, use_rht, False)
    dg = quantize_fast(wf.t().contiguous(), use_rht, False)
    if CACHE_WEIGHT_IMAGES:
        gemm_images(fp)
        gemm_images(dg)
    return FP4Weight(fp, dg, n, k, use_rht)


class FP4Linear(torch.autograd.Function):
    """fwd: Q(rht(x)) RN -> GEMM(fprop) -> x dtype; bwd: Q(rht(dy)) SR -> GEMM(dgrad); no weight
    grad (recant/model/nvfp4.py:151-170)."""

    @staticmethod
    def forward(ctx, x, w: FP4Weight):
        ctx.w = w
        x2 = x.reshape(-1, w.in_features)
        a = quantize_activation(x2, w.use_rht)
        y = _gemm_to(a, w.fprop, x.dtype)
        return y.reshape(*x.shape[:-1], w.out_features).to(x.dtype)

    @staticmethod
    def backward(ctx, dy):
        w = ctx.w
        d2 = dy.reshape(-1, w.out_features)
        d = quantize_activation(d2, w.use_rht, stochastic=True)
        dx = _gemm_to(d, w.dgrad, dy.dtype)
        return dx.reshape(*dy.shape[:-1], w.in_features).to(dy.dtype), None


def _gemm_to(a, b, dtype):
    """The selected GEMM backend; with this package's own backend and a bf16 activation the
    epilogue writes bf16 directly (one rounding of acc * gA * gB) instead of fp32 then a cast."""
    if _state["gemm"] == "b200" and dtype == torch.bfloat16:
        with torch.profiler.record_function("b:fp4_gemm"):
            return gemm_b200(a, b, out_dtype=torch.bfloat16)
    return gemm_fp4(a, b)


def fp4_linear(x: torch.Tensor, w: FP4Weight) -> torch.Tensor:
    return FP4Linear.apply(x, w)


# ----- registry mirror of recant/model/nvfp4.py:125-149 --------------------------------------
GEMM_BACKENDS = {"b200": gemm_b200}
_state = {"gemm": "b200"}
_fast = {"quantize": True}


def set_gemm_backend(name: str) -> None:
    if name not in GEMM_BACKENDS:
        raise KeyError(f"unknown FP4 GEMM backend {name!r}; have {list(GEMM_BACKENDS)}")
    _state["gemm"] = name


def get_gemm_backend() -> str:
    return _state["gemm"]


def gemm_fp4(a, b) -> torch.Tensor:
    with torch.profiler.record_function("b:fp4_gemm"):
        return GEMM_BACKENDS[_state["gemm"]](a, b)


def quantize_activation(x: torch.Tensor, use_rht: bool = True, stochastic: bool = False) -> FP4Tensor:
    with torch.profiler.record_function("b:quantize"):
        return quantize_fast(x.contiguous(), use_rht, stochastic)


def register(ref_nvfp4_module, select: bool = False, quantizer: bool = True) -> None:
    """Plug this package into the reference's ``recant.model.nvfp4`` module.

    * Adds ``'b200'`` to its ``GEMM_BACKENDS`` (nvfp4.py:125) and, with ``select``, makes it the
      active backend through ``set_gemm_backend`` (nvfp4.py:128-131).
    * With ``quantizer`` (the default), installs :func:`quantize_fast` as the fast quantizer hook:
      the reference's ``quantize_activation`` (nvfp4.py:144-149) calls
      ``fp4_kernels.quantize_fast(x, use_rht, stochastic)`` from its sibling module once
      ``_fast['quantize']`` is on, so this sets ``quantize_fast`` on that module (created as a
      plain module when the Triton one has not been imported, so Triton is never needed) and turns
      the switch on with ``set_fast_quantizer(True)`` (nvfp4.py:139-142)."""
    ref_nvfp4_module.GEMM_BACKENDS["b200"] = gemm_b200
    if select:
        ref_nvfp4_module.set_gemm_backend("b200")
    if quantizer:
        import sys
        import types
        pkg_name = ref_nvfp4_module.__name__.rpartition(".")[0]
        mod_name = (pkg_name + "." if pkg_name else "") + "fp4_kernels"
        mod = sys.modules.get(mod_name)
        if mod is None:
            mod = types.ModuleType(mod_name, "recant_b200 quantizer installed as the fast NVFP4 quantizer hook")
            sys.modules[mod_name] = mod
            pkg = sys.modules.get(pkg_name)
            if pkg is not None:
                setattr(pkg, "fp4_kernels", mod)
        mod.quantize_fast = quantize_fast
        ref_nvfp4_module.set_fast_quantizer(True)
