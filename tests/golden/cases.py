"""Seeded case recipes shared by the golden generator and the tests.

Inputs are regenerated from these recipes (torch CPU generators are deterministic), so the
fixtures store only the reference's outputs.
"""
from __future__ import annotations

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from oracle import inputs as I  # noqa: E402


def quantize_cases():
    """The reference self-check cases (recant/selfcheck.py:11-13) plus edge cases."""
    out, i = [], 0
    for dtype in ("bf16", "f32"):
        for m, k in ((300, 2048), (257, 6144), (17, 96)):
            for rot in (True, False):
                out.append(dict(name=f"sc{i}", kind="selfcheck", dtype=dtype, m=m, k=k, rht=rot, seed=100 + i))
                i += 1
    for dtype in ("bf16", "f32"):
        for rot in (True, False):
            out.append(dict(name=f"zero_{dtype}_{int(rot)}", kind="zeros", dtype=dtype, m=5, k=64, rht=rot, seed=0))
            out.append(dict(name=f"ties_{dtype}_{int(rot)}", kind="ties", dtype=dtype, m=3, k=32, rht=rot, seed=0))
            out.append(dict(name=f"tiny_{dtype}_{int(rot)}", kind="tiny", dtype=dtype, m=33, k=48, rht=rot, seed=5))
    out.append(dict(name="act_2048x4096", kind="normal", dtype="bf16", m=2048, k=4096, rht=True, seed=11))
    return out


_TD = {"bf16": torch.bfloat16, "f32": torch.float32}


def quantize_input(case) -> torch.Tensor:
    gen = torch.Generator().manual_seed(case["seed"])
    m, k = case["m"], case["k"]
    kind = case["kind"]
    if kind == "selfcheck":
        x = torch.randn(m, k, generator=gen) * 3
        x[:, ::37] *= 30
    elif kind == "zeros":
        x = torch.zeros(m, k)
    elif kind == "ties":
        # block maxima of 6 and values on every rounding midpoint, both signs
        row = torch.tensor([6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0,
                            -0.25, -0.75, -2.5, -5.0, -0.1, 0.1, 3.0, -6.0])
        x = torch.stack([row.repeat(k // 16), row.flip(0).repeat(k // 16) * 0.5,
                         row.repeat(k // 16) * 1e-3])[:m]
    elif kind == "tiny":
        # wide dynamic range so some per-16 scales land in e4m3 subnormals / zero
        x = torch.randn(m, k, generator=gen) * torch.logspace(-8, 2, k).unsqueeze(0)
    else:
        x = torch.randn(m, k, generator=gen)
    return x.to(_TD[case["dtype"]]).contiguous()


def weight_cases():
    return [dict(name="w256x96", n=256, k=96, seed=21), dict(name="w512x256", n=512, k=256, seed=22)]


def weight_input(case) -> torch.Tensor:
    gen = torch.Generator().manual_seed(case["seed"])
    return torch.randn(case["n"], case["k"], generator=gen) * 0.02


def gemm_cases():
    return [dict(name="g40x96x256", m=40, n=256, k=96, seed=31)]


def gemm_input(case):
    gen = torch.Generator().manual_seed(case["seed"])
    x = torch.randn(case["m"], case["k"], generator=gen)
    w = torch.randn(case["n"], case["k"], generator=gen) * 0.05
    return x, w


def gdn_cases():
    return [
        # config-0 gate distribution, ragged T (3 chunks, last one partial), GQA 1->2, h0, dht
        dict(name="gdn_ragged", B=2, T=130, Hk=1, Hv=2, d=128, seed=0, mild=False, h0=True),
        # slowly-decaying gates (the reference's select_gdn check uses g = -U(0, 0.1))
        dict(name="gdn_mild", B=1, T=192, Hk=2, Hv=2, d=128, seed=3, mild=True, h0=False),
    ]


def gdn_input(case):
    inp = I.gdn_inputs(case["B"], case["T"], case["Hk"], case["Hv"], case["d"], dtype=torch.float32,
                       seed=case["seed"])
    gen = torch.Generator().manual_seed(case["seed"] + 1000)
    if case["mild"]:
        inp["g"] = -torch.rand(case["B"], case["T"], case["Hv"], generator=gen) * 0.1
    do = I.grad_output(case["B"], case["T"], case["Hv"], case["d"], dtype=torch.float32, seed=case["seed"] + 1)
    shape = (case["B"], case["Hv"], case["d"], case["d"])
    h0 = torch.randn(*shape, generator=gen) * 0.1 if case["h0"] else None
    dht = torch.randn(*shape, generator=gen) * 0.1
    return inp, do, h0, dht
