"""Chunked Gated DeltaNet op on B200, shaped like the reference backend registry.

Drop-in for ``recant.model.ops``'s GDN backends (recant/model/ops.py:5-10,56-67):

* :func:`gdn_b200` has the signature of ``gdn_torch``/``gdn_fla``
  ``fn(q, k, v, g, beta, initial_state=None, output_final_state=False) -> (o, final_state|None)``
  and the semantics of ``gdn_torch`` (qk L2-norm and dk^-0.5 inside the op, chunk 64, fp32 state,
  o in the input dtype); its backward is a ``torch.autograd.Function`` giving dq, dk, dv, dg,
  dbeta and d(initial_state).
* Extensions (defaults keep every reference call site unchanged): ``cu_seqlens`` (int64 [N+1],
  B == 1, per-sequence state reset, the fla varlen convention), q/k with Hk < Hv heads (GQA
  without repeat_interleave), ``scale`` and ``path`` ("auto" | "exact" | "fast" | "recurrent").
* :func:`gdn_recurrent`: the token-by-token forward of the decode step (short calls with a carried
  state and no gradient), chosen automatically by ``gdn_b200`` for such calls.
* :data:`GDN_BACKENDS`, :func:`set_gdn_backend`, :func:`get_gdn_backend`, :func:`gdn_core` mirror
  ops.py's registry; :func:`register` adds ``'b200'`` to the reference's own registry.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L

_PATHS = {"auto": L.GDN_AUTO, "exact": L.GDN_EXACT, "fast": L.GDN_FAST}
_DT = {torch.float32: L.F32, torch.bfloat16: L.BF16}


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _Problem:
    def __init__(self, q, k, v, g, beta, initial_state, cu_seqlens, scale, path):
        if not q.is_cuda:
            raise ValueError("recant_b200.gdn: inputs must be CUDA tensors (no CPU path)")
        if q.dim() != 4 or k.shape != q.shape or v.dim() != 4:
            raise ValueError(f"recant_b200.gdn: q/k must be [B,T,Hk,dk] and v [B,T,Hv,dv]; got "
                             f"{tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
        B, T, Hk, dk = q.shape
        Hv, dv = v.shape[2], v.shape[3]
        if v.shape[:2] != (B, T) or g.shape != (B, T, Hv) or beta.shape != (B, T, Hv):
            raise ValueError("recant_b200.gdn: g and beta must be [B,T,Hv] matching v")
        if q.dtype not in _DT:
            raise TypeError(f"recant_b200.gdn: dtype {q.dtype} unsupported (float32 or bfloat16)")
        self.dtype = q.dtype
        self.B, self.T, self.Hk, self.Hv, self.dk, self.dv = B, T, Hk, Hv, dk, dv
        if cu_seqlens is not None:
            if B != 1:
                raise ValueError("recant_b200.gdn: cu_seqlens requires B == 1")
            self.n_seqs = cu_seqlens.numel() - 1
        else:
            self.n_seqs = B
        if initial_state is not None and initial_state.shape != (self.n_seqs, Hv, dk, dv):
            raise ValueError(f"recant_b200.gdn: initial_state must be [{self.n_seqs},{Hv},{dk},{dv}]")
        self.scale = float(dk ** -0.5 if scale is None else scale)
        self.path = _PATHS[path]
        saved, scratch = C.c_size_t(0), C.c_size_t(0)
        L.check(L.lib().rb2_gdn_workspace_split(B, T, self.n_seqs, Hk, Hv, dk, dv, _DT[q.dtype], self.path,
                                                C.byref(saved), C.byref(scratch)), "gdn_workspace_split")
        # the forward keeps only the saved part alive until the backward; the backward-only
        # scratch is allocated inside the backward (the caching allocator recycles it)
        self.ws_bytes, self.scratch_bytes = saved.value, scratch.value

    def args(self):
        return (self.B, self.T, self.n_seqs, self.Hk, self.Hv, self.dk, self.dv, _DT[self.dtype], self.path,
                self.scale)


class _GDNFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, initial_state, cu_seqlens, output_final_state, scale, path):
        pb = _Problem(q, k, v, g, beta, initial_state, cu_seqlens, scale, path)
        dt = pb.dtype
        q, k, v = (t.contiguous() for t in (q, k, v))
        g = g.to(torch.float32).contiguous()
        beta_k = beta.to(dt).contiguous()
        h0 = None if initial_state is None else initial_state.to(torch.float32).contiguous()
        cu = None if cu_seqlens is None else cu_seqlens.to(device=q.device, dtype=torch.int64).contiguous()
        ws = torch.empty(pb.ws_bytes, dtype=torch.uint8, device=q.device)
        o = torch.empty(pb.B, pb.T, pb.Hv, pb.dv, dtype=dt, device=q.device)
        hT = torch.empty(pb.n_seqs, pb.Hv, pb.dk, pb.dv, dtype=torch.float32, device=q.device)
        st = L.lib().rb2_gdn_fwd(L.ptr(q), L.ptr(k), L.ptr(v), L.ptr(g), L.ptr(beta_k), L.ptr(h0), L.ptr(cu),
                                 *pb.args(), L.ptr(o), L.ptr(hT), L.ptr(ws), pb.ws_bytes, _stream(q.device))
        L.check(st, "gdn_fwd")
        L.check_status(ws, "gdn_fwd")
        ctx.set_materialize_grads(False)  # an unused final state needs no zero gradient
        ctx.save_for_backward(q, k, v, g, beta_k, h0, cu)
        ctx.pb, ctx.ws = pb, ws
        ctx.beta_dtype = beta.dtype
        ctx.has_h0 = initial_state is not None
        return o, hT

    @staticmethod
    def backward(ctx, do, dhT):
        q, k, v, g, beta, h0, cu = ctx.saved_tensors
        pb, ws = ctx.pb, ctx.ws
        if do is None:
            do = torch.zeros(pb.B, pb.T, pb.Hv, pb.dv, dtype=pb.dtype, device=q.device)
        do = do.to(pb.dtype).contiguous()
        dhT = None if dhT is None else dhT.to(torch.float32).contiguous()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        dg = torch.empty_like(g)
        dbeta = torch.empty_like(beta)
        dh0 = torch.empty_like(h0) if ctx.has_h0 and ctx.needs_input_grad[5] else None
        scratch = torch.empty(max(pb.scratch_bytes, 1), dtype=torch.uint8, device=q.device)
        st = L.lib().rb2_gdn_bwd_ex(L.ptr(q), L.ptr(k), L.ptr(v), L.ptr(g), L.ptr(beta), L.ptr(h0), L.ptr(cu),
                                    *pb.args(), L.ptr(do), L.ptr(dhT), L.ptr(dq), L.ptr(dk), L.ptr(dv), L.ptr(dg),
                                    L.ptr(dbeta), L.ptr(dh0), L.ptr(ws), pb.ws_bytes, L.ptr(scratch),
                                    pb.scratch_bytes, _stream(q.device), 3, 0)
        L.check(st, "gdn_bwd")
        L.check_status(ws, "gdn_bwd")
        return dq, dk, dv, dg, dbeta.to(ctx.beta_dtype), dh0, None, None, None, None


# Calls of at most this many tokens that need no gradient (the decode step) take the recurrent kernel
RECURRENT_MAX_T = 16


def _needs_grad(*ts):
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts)


def gdn_recurrent(q, k, v, g, beta, initial_state=None, output_final_state=False, *, cu_seqlens=None, scale=None,
                  final_state_out=None):
    """Forward only, token by token, with a carried fp32 state: the decode step (layers.py:177-180 under
    serve/engine.py:107-119). Same contract and arithmetic as gdn_torch on one padded chunk
    (ops.py:21-54); no autograd graph. ``final_state_out``: a contiguous fp32 [n_seqs, Hv, dk, dv]
    tensor to receive the final state (it may be ``initial_state`` itself: updated in place)."""
    if not q.is_cuda:
        raise ValueError("recant_b200.gdn: inputs must be CUDA tensors (no CPU path)")
    if q.dim() != 4 or k.shape != q.shape or v.dim() != 4:
        raise ValueError(f"recant_b200.gdn: q/k must be [B,T,Hk,dk] and v [B,T,Hv,dv]; got "
                         f"{tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    B, T, Hk, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    if v.shape[:2] != (B, T) or g.shape != (B, T, Hv) or beta.shape != (B, T, Hv):
        raise ValueError("recant_b200.gdn: g and beta must be [B,T,Hv] matching v")
    if q.dtype not in _DT:
        raise TypeError(f"recant_b200.gdn: dtype {q.dtype} unsupported (float32 or bfloat16)")
    n_seqs = B if cu_seqlens is None else cu_seqlens.numel() - 1
    if initial_state is not None and initial_state.shape != (n_seqs, Hv, dk, dv):
        raise ValueError(f"recant_b200.gdn: initial_state must be [{n_seqs},{Hv},{dk},{dv}]")
    dt = q.dtype
    q, k, v = (t.detach().contiguous() for t in (q, k, v))
    g = g.detach().to(torch.float32).contiguous()
    beta_k = beta.detach().to(dt).contiguous()
    h0 = None if initial_state is None else initial_state.detach().to(torch.float32).contiguous()
    cu = None if cu_seqlens is None else cu_seqlens.to(device=q.device, dtype=torch.int64).contiguous()
    o = torch.empty(B, T, Hv, dv, dtype=dt, device=q.device)
    if final_state_out is not None:
        if (final_state_out.shape != (n_seqs, Hv, dk, dv) or final_state_out.dtype != torch.float32
                or not final_state_out.is_contiguous()):
            raise ValueError("recant_b200.gdn_recurrent: final_state_out must be a contiguous fp32 "
                             f"[{n_seqs},{Hv},{dk},{dv}] tensor")
        hT = final_state_out
    else:
        hT = torch.empty(n_seqs, Hv, dk, dv, dtype=torch.float32, device=q.device) if output_final_state else None
    sc = float(dk ** -0.5 if scale is None else scale)
    L.check(L.lib().rb2_gdn_recurrent_fwd(L.ptr(q), L.ptr(k), L.ptr(v), L.ptr(g), L.ptr(beta_k), L.ptr(h0),
                                          L.ptr(cu), B, T, n_seqs, Hk, Hv, dk, dv, _DT[dt], sc, L.ptr(o), L.ptr(hT),
                                          _stream(q.device)), "gdn_recurrent_fwd")
    return o, hT


def gdn_b200(q, k, v, g, beta, initial_state=None, output_final_state=False, *, cu_seqlens=None,
             scale=None, path="auto"):
    """GDN on B200 with gdn_torch's contract (recant/model/ops.py:21-54): the chunked op, or for a
    call of at most RECURRENT_MAX_T tokens that needs no gradient (``path="auto"``), or always with
    ``path="recurrent"``, the token-by-token forward. That kernel builds no autograd graph, so
    ``path="recurrent"`` on inputs that need a gradient raises ValueError instead of silently
    returning an output that gradients cannot flow through."""
    needs_grad = _needs_grad(q, k, v, g, beta, initial_state)
    if path == "recurrent" and needs_grad:
        raise ValueError("recant_b200.gdn_b200: path='recurrent' is forward-only and the inputs require grad; "
                         "use path='auto' or 'fast' for training, or call it under torch.no_grad()")
    if path == "recurrent" or (path == "auto" and q.shape[1] <= RECURRENT_MAX_T and not needs_grad):
        o, hT = gdn_recurrent(q, k, v, g, beta, initial_state, output_final_state, cu_seqlens=cu_seqlens,
                              scale=scale)
        return o, (hT if output_final_state else None)
    o, hT = _GDNFunction.apply(q, k, v, g, beta, initial_state, cu_seqlens, output_final_state, scale, path)
    return o, (hT if output_final_state else None)


# ----- registry mirror of recant/model/ops.py:5-10,60-67 -------------------------------------
GDN_BACKENDS = {"b200": gdn_b200}
_state = {"gdn": "b200"}


def set_gdn_backend(name: str) -> None:
    if name not in GDN_BACKENDS:
        raise KeyError(f"unknown GDN backend {name!r}; have {list(GDN_BACKENDS)}")
    _state["gdn"] = name


def get_gdn_backend() -> str:
    return _state["gdn"]


def gdn_core(q, k, v, g, beta, initial_state=None, output_final_state=False):
    with torch.profiler.record_function("b:gdn"):
        return GDN_BACKENDS[_state["gdn"]](q, k, v, g, beta, initial_state=initial_state,
                                           output_final_state=output_final_state)


def register(ref_ops_module, select: bool = False) -> None:
    """Add ``'b200'`` to the reference's ``ops.GDN_BACKENDS`` (and optionally select it)."""
    ref_ops_module.GDN_BACKENDS["b200"] = gdn_b200
    if select:
        ref_ops_module.set_gdn_backend("b200")
