"""Chunked Gated DeltaNet oracle on the CPU -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates the reference op ``recant.model.ops.gdn_torch`` (recant/model/ops.py:21-54) with
torch CPU ops, and takes its backward from autograd exactly as the reference does (the
reference has no hand-written backward; ``FP4Linear``-free GDN grads come from autograd over
this graph, ops.py:21-54 via layers.py:178 and branch.py:208-219).

Algorithm (per head, chunk size C=64, all in ``dtype``, fp32 by default as ops.py:25):
  q, k <- l2norm(q), l2norm(k) with eps 1e-6 inside the rsqrt (ops.py:18-19,26); q *= dk^-1/2
  (ops.py:27); zero-pad T to a multiple of C (ops.py:28-31).
  Within a chunk: cum = cumsum(g); Gam_ij = exp(cum_i - cum_j) for i >= j else 0 (ops.py:35-37)
    A_kk = (beta k) k^T * Gam   (only the strict lower part matters, ops.py:38)
    A_qk = q k^T * Gam          (ops.py:39)
    U = (I + A_kk)^-1 (beta v),  W = (I + A_kk)^-1 (beta k * e^cum)  (unit-lower solve, ops.py:40-42)
    q~ = q e^cum, k~ = k e^(cum_last - cum), gamma = e^cum_last        (ops.py:45-47)
  Across chunks (sequential, ops.py:49-52):
    V' = U - W S;  O = q~ S + A_qk V';  S <- gamma S + k~^T V'
  o is cast back to the input dtype, the state stays fp32 (ops.py:53-54).

Extensions the B200 op adds (absent in the reference op, so restated through it):
  * GQA: q, k with Hk < Hv heads are repeated to Hv first, as the reference caller does
    (recant/model/layers.py:174-176);
  * cu_seqlens (B == 1): each segment runs independently from its own initial state, which is
    the fla varlen convention; the oracle loops the single-sequence op per segment.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

CHUNK = 64


def _unit_norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).sum(-1, keepdim=True) + eps)


def gdn_forward(q, k, v, g, beta, initial_state=None, output_final_state=False,
                chunk: int = CHUNK, dtype=torch.float32):
    """Single-batch-layout chunked GDN. q,k [B,T,H,dk]; v [B,T,H,dv]; g,beta [B,T,H].

    Differentiable (autograd) in every input, as the reference op is.
    """
    out_dtype = q.dtype
    B, T, H, dk = k.shape
    dv = v.shape[-1]
    if T == 0:  # an empty segment passes its state through unchanged
        S = torch.zeros(B, H, dk, dv, dtype=dtype) if initial_state is None else initial_state.to(dtype)
        o = torch.zeros(B, 0, H, dv, dtype=out_dtype) + 0.0 * S.sum()
        return o, (S.to(torch.float32) if output_final_state else None)
    # head-major working layout [B, H, T, d]
    qh, kh, vh = (t.permute(0, 2, 1, 3).to(dtype) for t in (q, k, v))
    bh, gh = (t.permute(0, 2, 1).to(dtype) for t in (beta, g))
    qh = _unit_norm(qh) * (dk ** -0.5)
    kh = _unit_norm(kh)
    pad = (-T) % chunk
    if pad:
        qh, kh, vh = (F.pad(t, (0, 0, 0, pad)) for t in (qh, kh, vh))
        bh, gh = (F.pad(t, (0, pad)) for t in (bh, gh))
    n = (T + pad) // chunk
    split = lambda t: t.reshape(B, H, n, chunk, *t.shape[3:])
    qc, kc, vc, bc, gc = (split(t) for t in (qh, kh, vh, bh, gh))
    cum = gc.cumsum(-1)                                            # [B,H,n,C]
    causal = torch.ones(chunk, chunk, dtype=torch.bool).tril()
    gam = torch.where(causal, (cum[..., :, None] - cum[..., None, :]), float("-inf")).exp()
    kb = kc * bc[..., None]
    a_kk = (kb @ kc.transpose(-1, -2)) * gam
    a_qk = (qc @ kc.transpose(-1, -2)) * gam
    ecum = cum.exp()[..., None]
    u = torch.linalg.solve_triangular(a_kk, vc * bc[..., None], upper=False, unitriangular=True)
    w = torch.linalg.solve_triangular(a_kk, kb * ecum, upper=False, unitriangular=True)
    q_dec = qc * ecum
    k_dec = kc * (cum[..., -1:] - cum).exp()[..., None]
    gamma = cum[..., -1].exp()[..., None, None]                    # [B,H,n,1,1]
    if initial_state is None:
        S = torch.zeros(B, H, dk, dv, dtype=dtype)
    else:
        S = initial_state.to(dtype)
    outs = []
    for c in range(n):
        v_new = u[:, :, c] - w[:, :, c] @ S
        outs.append(q_dec[:, :, c] @ S + a_qk[:, :, c] @ v_new)
        S = gamma[:, :, c] * S + k_dec[:, :, c].transpose(-1, -2) @ v_new
    o = torch.stack(outs, 2).reshape(B, H, n * chunk, dv)[:, :, :T]
    o = o.permute(0, 2, 1, 3).contiguous().to(out_dtype)
    return o, (S.to(torch.float32) if output_final_state else None)


def expand_heads(x: torch.Tensor, hv: int) -> torch.Tensor:
    """GQA: repeat each of Hk heads Hv/Hk times along dim 2 (layers.py:174-176)."""
    hk = x.shape[2]
    return x if hk == hv else x.repeat_interleave(hv // hk, dim=2)


def gdn(q, k, v, g, beta, initial_state=None, output_final_state=False, cu_seqlens=None,
        dtype=torch.float32):
    """The B200 op's contract on the CPU: GQA-aware, optional cu_seqlens (B must be 1)."""
    hv = v.shape[2]
    q, k = expand_heads(q, hv), expand_heads(k, hv)
    if cu_seqlens is None:
        return gdn_forward(q, k, v, g, beta, initial_state, output_final_state, dtype=dtype)
    assert q.shape[0] == 1, "cu_seqlens requires B == 1"
    cu = [int(x) for x in cu_seqlens]
    outs, finals = [], []
    for i in range(len(cu) - 1):
        s, e = cu[i], cu[i + 1]
        h0 = None if initial_state is None else initial_state[i:i + 1]
        o, st = gdn_forward(q[:, s:e], k[:, s:e], v[:, s:e], g[:, s:e], beta[:, s:e], h0,
                            output_final_state, dtype=dtype)
        outs.append(o)
        finals.append(st)
    o = torch.cat(outs, 1)
    return o, (torch.cat(finals, 0) if output_final_state else None)


def gdn_fwd_bwd(q, k, v, g, beta, do, initial_state=None, dht=None, cu_seqlens=None,
                dtype=torch.float32):
    """Forward plus autograd backward. Returns (o, hT, grads dict) with grads for
    q, k, v, g, beta and initial_state (when given)."""
    leaves = {n: t.detach().clone().requires_grad_(True)
              for n, t in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta))}
    h0 = None
    if initial_state is not None:
        h0 = initial_state.detach().clone().requires_grad_(True)
        leaves["h0"] = h0
    want = dht is not None
    o, hT = gdn(leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["beta"], h0,
                output_final_state=True, cu_seqlens=cu_seqlens, dtype=dtype)
    loss = (o.float() * do.float()).sum()
    if want:
        loss = loss + (hT * dht.float()).sum()
    else:
        loss = loss + 0.0 * hT.sum()
    loss.backward()
    grads = {n: t.grad for n, t in leaves.items()}
    return o.detach(), hT.detach(), grads
