"""GDN parity on the GPU: CUDA library vs the CPU oracle / the reference's golden outputs.

Tolerances (relative Frobenius): 1e-4 for fp32 inputs (exact path) and 2e-2 for bf16 inputs
against the fp32 reference, as the benchmark contract states.
"""
import os

import numpy as np
import pytest
import torch

import cases
from gpu_util import rel, run_b200
from oracle import gdn as OG
from oracle import inputs as I

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_arrays.npz"))
F32_TOL = 1e-4
BF16_TOL = 2e-2


def _compare(o, hT, gr, ref_o, ref_hT, ref_gr, tol, names=("q", "k", "v", "g", "beta")):
    errs = {"o": rel(o, ref_o), "hT": rel(hT, ref_hT)}
    for n in names:
        errs["d" + n] = rel(gr[n], ref_gr[n])
    if "h0" in ref_gr and ref_gr["h0"] is not None:
        errs["dh0"] = rel(gr["h0"], ref_gr["h0"])
    bad = {k: v for k, v in errs.items() if not v < tol}
    assert not bad, f"over tolerance {tol}: {bad} (all: {errs})"
    return errs


@pytest.mark.parametrize("case", cases.gdn_cases(), ids=lambda c: c["name"])
def test_exact_path_matches_reference_golden(case):
    inp, do, h0, dht = cases.gdn_input(case)
    o, hT, gr = run_b200(inp, do, h0, dht, path="exact")
    nm = case["name"]
    ref = {n: torch.from_numpy(GOLD[f"{nm}_d{n}"]) for n in ("q", "k", "v", "g", "beta")}
    if h0 is not None:
        ref["h0"] = torch.from_numpy(GOLD[f"{nm}_dh0"])
    _compare(o, hT, gr, torch.from_numpy(GOLD[f"{nm}_o"]), torch.from_numpy(GOLD[f"{nm}_hT"]), ref, F32_TOL)


def test_config0_fp32_parity():
    """Config 0 (B1 T1024 Hk4 Hv8 d128, fp32): <= 1e-4 against the fp32 reference, fwd + bwd."""
    inp = I.gdn_inputs(1, 1024, 4, 8, 128, dtype=torch.float32, seed=0)
    do = I.grad_output(1, 1024, 8, 128, dtype=torch.float32)
    ro, rhT, rg = OG.gdn_fwd_bwd(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], do)
    o, hT, gr = run_b200(inp, do, path="exact")
    _compare(o, hT, gr, ro, rhT, rg, F32_TOL)


@pytest.mark.parametrize("T", [1, 63, 64, 65, 200])
def test_ragged_lengths_fp32(T):
    inp = I.gdn_inputs(2, T, 2, 4, 128, dtype=torch.float32, seed=T)
    do = I.grad_output(2, T, 4, 128, dtype=torch.float32, seed=T + 1)
    gen = torch.Generator().manual_seed(T)
    h0 = torch.randn(2, 4, 128, 128, generator=gen) * 0.1
    dht = torch.randn(2, 4, 128, 128, generator=gen) * 0.1
    ro, rhT, rg = OG.gdn_fwd_bwd(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], do, h0, dht)
    o, hT, gr = run_b200(inp, do, h0, dht, path="exact")
    _compare(o, hT, gr, ro, rhT, rg, F32_TOL)


def test_varlen_fp32_matches_per_sequence_oracle():
    lengths = [70, 1, 64, 0, 129, 33]
    cu = I.cu_seqlens_of(lengths)
    T = int(cu[-1])
    inp = I.gdn_inputs(1, T, 2, 4, 128, dtype=torch.float32, seed=5)
    do = I.grad_output(1, T, 4, 128, dtype=torch.float32, seed=6)
    gen = torch.Generator().manual_seed(7)
    h0 = torch.randn(len(lengths), 4, 128, 128, generator=gen) * 0.1
    dht = torch.randn(len(lengths), 4, 128, 128, generator=gen) * 0.1
    ro, rhT, rg = OG.gdn_fwd_bwd(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], do, h0, dht, cu_seqlens=cu)
    o, hT, gr = run_b200(inp, do, h0, dht, cu=cu, path="exact")
    _compare(o, hT, gr, ro, rhT, rg, F32_TOL)


@pytest.mark.parametrize("path", ["auto", "exact"])
def test_bf16_inputs_within_2e2(path):
    """bf16 inputs vs the fp32 reference on the same (bf16-representable) values."""
    inp = I.gdn_inputs(2, 300, 2, 4, 128, dtype=torch.bfloat16, seed=11)
    do = I.grad_output(2, 300, 4, 128, dtype=torch.bfloat16, seed=12)
    f32 = {n: t.float() for n, t in inp.items()}
    ro, rhT, rg = OG.gdn_fwd_bwd(f32["q"], f32["k"], f32["v"], f32["g"], f32["beta"], do.float())
    o, hT, gr = run_b200(inp, do, path=path)
    _compare(o, hT, gr, ro, rhT, rg, BF16_TOL)


def test_reference_select_gdn_check():
    """The reference's own backend check (recant/backends.py:51-65): bf16, b1 t512 h32 d128,
    g = -U(0, 0.1), beta = U(0, 1): rel err < 0.05 and finite q.grad."""
    gen = torch.Generator().manual_seed(0)
    b, t, h = 1, 512, 32
    mk = lambda *s: torch.randn(*s, generator=gen).to(torch.bfloat16)
    q, k, v = mk(b, t, h, 128), mk(b, t, h, 128), mk(b, t, h, 128)
    g = -torch.rand(b, t, h, generator=gen) * 0.1
    beta = torch.rand(b, t, h, generator=gen).to(torch.bfloat16)
    o_ref, _ = OG.gdn(q.float(), k.float(), v.float(), g, beta.float())
    inp = dict(q=q, k=k, v=v, g=g, beta=beta)
    o, hT, gr = run_b200(inp, torch.ones(b, t, h, 128, dtype=torch.bfloat16))
    assert rel(o, o_ref) < 0.05 and torch.isfinite(gr["q"]).all()


def test_deterministic():
    inp = I.gdn_inputs(1, 256, 2, 4, 128, dtype=torch.bfloat16, seed=3)
    do = I.grad_output(1, 256, 4, 128, dtype=torch.bfloat16, seed=4)
    a = run_b200(inp, do)
    b = run_b200(inp, do)
    assert torch.equal(a[0], b[0]) and all(torch.equal(a[2][n], b[2][n]) for n in a[2])
