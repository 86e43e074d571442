"""Affine segment hand-off on the CPU -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The reference op walks one sequence's chunks in order (recant/model/ops.py:49-52):
S <- gamma S + k~^T (U - W S). Each step is affine in S, so a run of chunks maps
S_out = M S_in + c (M = product of (gamma I - k~^T W), c = S_out for S_in = 0), and the backward
maps dS_in = M^T dS_out + d. These plain torch loops restate the folds that the segmented and
context-parallel op runs with its fold kernel; the tests check them against the unsegmented
oracle (oracle.gdn), and the kernel against them.
"""
from __future__ import annotations

import torch


def fold(Ms, cs, s0, transpose=False):
    """Values entering each map and the value after the last one.
    forward: x_0 = s0, x_{k+1} = M_k x_k + c_k; transposed: from k = n-1 down, x = M_k^T x + c_k."""
    n = Ms.shape[0]
    order = range(n - 1, -1, -1) if transpose else range(n)
    x = s0
    states = [None] * n
    for k in order:
        states[k] = x
        A = Ms[k].transpose(-1, -2) if transpose else Ms[k]
        x = A @ x + (cs[k] if cs is not None else 0)
    return (torch.stack(states, 0) if n else Ms[:0].clone()), x


def compose(Ms, cs):
    """(M_{n-1} ... M_0, fold of c from zero) for maps applied in order 0..n-1."""
    eye = torch.eye(Ms.shape[-1], dtype=Ms.dtype).expand_as(Ms[0]).clone()
    _, M = fold(Ms, None, eye)
    _, c = fold(Ms, cs, torch.zeros_like(cs[0]))
    return M, c


def prefix(Ms, cs, s0):
    """S_in of every segment: S_in[0] = s0, S_in[k] = M[k-1] S_in[k-1] + c[k-1]."""
    return fold(Ms, cs, s0)[0]


def suffix(Ms, ds, d_last):
    """dS_out of every segment: dS_out[n-1] = d_last, dS_out[k] = M[k+1]^T dS_out[k+1] + ds[k+1]."""
    return fold(Ms, ds, d_last, transpose=True)[0]


def rank_input_state(M_all, c_all, rank, s0):
    """The state entering ``rank``'s shard: ranks 0..rank-1's composed maps folded onto s0."""
    return fold(M_all[:rank], c_all[:rank], s0)[1]


def rank_output_grad(M_all, d_all, rank, d_final):
    """The gradient of the state leaving ``rank``'s shard: ranks world-1..rank+1 folded
    (transposed) onto the gradient of the sequence's final state."""
    return fold(M_all[rank + 1:], d_all[rank + 1:], d_final, transpose=True)[1]
