"""Pin the CPU oracle to the reference's own outputs (fixtures from tests/golden/make_golden.py)."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import cases
from oracle import gdn as OG
from oracle import nvfp4 as ON

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


with open(os.path.join(GOLD, "nvfp4_golden.json")) as f:
    NV = json.load(f)
ARR = np.load(os.path.join(GOLD, "golden_arrays.npz"))


@pytest.mark.parametrize("case", NV["quantize"], ids=lambda c: c["name"])
def test_quantize_oracle_bit_exact(case):
    x = cases.quantize_input(case).float().numpy()
    codes, scales, gs = ON.quantize_activation(x, case["dtype"], case["rht"])
    assert _sha(codes) == case["codes"]
    assert _sha(scales) == case["scales"]
    assert _sha(ON.to_blocked(scales)) == case["blocked"]
    assert float(gs).hex() == case["gscale"]


@pytest.mark.parametrize("case", NV["weights"], ids=lambda c: c["name"])
def test_quantize_weight_oracle_bit_exact(case):
    w = cases.weight_input(case).numpy()
    fp, dg = ON.quantize_weight(w)
    assert _sha(fp[0]) == case["fprop_codes"] and _sha(fp[1]) == case["fprop_scales"]
    assert _sha(dg[0]) == case["dgrad_codes"] and _sha(dg[1]) == case["dgrad_scales"]
    assert float(fp[2]).hex() == case["fprop_gscale"] and float(dg[2]).hex() == case["dgrad_gscale"]


@pytest.mark.parametrize("case", NV["gemm"], ids=lambda c: c["name"])
def test_gemm_emulated_oracle(case):
    x, w = cases.gemm_input(case)
    a = ON.quantize_activation(x.numpy(), "f32", True) + ((case["m"], case["k"]),)
    fp, _ = ON.quantize_weight(w.numpy())
    y = ON.gemm_emulated(a, fp)
    ref = ARR[f"gemm_{case['name']}"]
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-6


def test_stochastic_rounding_unbiased():
    """SR parity is statistical (recant/selfcheck.py:22-27): mean of 64 draws within 3%."""
    gen = torch.Generator().manual_seed(4)
    x = (torch.randn(64, 256, generator=gen) * 2).to(torch.bfloat16).float().numpy()
    target = ON.rht(x, "bf16")
    rng = np.random.default_rng(0)
    acc = np.zeros_like(target)
    for _ in range(64):
        c, s, g = ON.quantize(target, stochastic=True, rng=rng)
        acc += ON.dequant(c, s, g, 256)
    acc /= 64
    assert np.abs(acc - target).mean() / np.abs(target).mean() < 0.03


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


@pytest.mark.parametrize("case", cases.gdn_cases(), ids=lambda c: c["name"])
def test_gdn_oracle_matches_reference(case):
    inp, do, h0, dht = cases.gdn_input(case)
    o, hT, gr = OG.gdn_fwd_bwd(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], do, h0, dht)
    nm = case["name"]
    assert _rel(o, ARR[f"{nm}_o"]) < 1e-6
    assert _rel(hT, ARR[f"{nm}_hT"]) < 1e-6
    for n in ("q", "k", "v", "g", "beta"):
        assert _rel(gr[n], ARR[f"{nm}_d{n}"]) < 1e-5, n
    if h0 is not None:
        assert _rel(gr["h0"], ARR[f"{nm}_dh0"]) < 1e-5


def test_gdn_oracle_varlen_equals_per_sequence():
    """cu_seqlens semantics: each packed segment equals the op run on that segment alone."""
    inp = cases.I.gdn_inputs(1, 200, 1, 2, 128, dtype=torch.float32, seed=9)
    cu = torch.tensor([0, 70, 71, 200])
    o, hT = OG.gdn(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], None, True, cu_seqlens=cu)
    for i in range(3):
        s, e = int(cu[i]), int(cu[i + 1])
        oi, hi = OG.gdn(*(inp[n][:, s:e] for n in ("q", "k", "v", "g", "beta")), None, True)
        assert torch.equal(o[:, s:e], oi) and torch.equal(hT[i:i + 1], hi)


def test_varlen_config3_token_count():
    assert sum(cases.I.varlen_lengths()) == 243613
