"""Seeded synthetic inputs for the benchmark configs -- TEST INFRASTRUCTURE ONLY.

The reference publishes no benchmark data; these generators reproduce the input
distributions the benchmark configs name (q, k ~ N(0,1) then L2-normalised inside the op;
v ~ N(0,1); beta = sigmoid(N(0,1)); g = -exp(A_log) * softplus(a) with A_log = log U(1,16)
per head and a ~ N(0,1), the gate of recant/model/fused_ops.py:32-33 with dt_bias = 0;
dO ~ N(0,1) from seed 1).  Draw order is fixed so every consumer sees the same tensors.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

CONFIGS = {
    # name: (B, T, Hk, Hv, d)
    "cfg0": (1, 1024, 4, 8, 128),
    "cfg1": (4, 4096, 16, 32, 128),
}


def gdn_inputs(B, T, Hk, Hv, d=128, dtype=torch.bfloat16, seed=0, device="cpu"):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, Hk, d, generator=gen)
    k = torch.randn(B, T, Hk, d, generator=gen)
    v = torch.randn(B, T, Hv, d, generator=gen)
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=gen))
    a_log = torch.log(torch.empty(Hv).uniform_(1.0, 16.0, generator=gen))
    a = torch.randn(B, T, Hv, generator=gen)
    g = -a_log.exp() * F.softplus(a)
    cast = lambda t: t.to(dtype).to(device)
    return dict(q=cast(q), k=cast(k), v=cast(v), g=g.float().to(device), beta=cast(beta))


def grad_output(B, T, Hv, d=128, dtype=torch.bfloat16, seed=1, device="cpu"):
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(B, T, Hv, d, generator=gen).to(dtype).to(device)


def varlen_lengths(n=64, lo=128, hi=8192, seed=0):
    """Config 3: 64 sequence lengths uniform in [128, 8192] (243,613 tokens at seed 0)."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=gen).tolist()


def cu_seqlens_of(lengths):
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + int(n))
    return torch.tensor(cu, dtype=torch.int64)
