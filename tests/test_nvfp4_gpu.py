"""NVFP4 quantizer parity on the GPU: bit-exact codes / scales / blocked scales / gscale against
the reference's own outputs (sha256 fixtures) and the numpy oracle."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import cases
from oracle import nvfp4 as ON

pytestmark = pytest.mark.gpu

with open(os.path.join(os.path.dirname(__file__), "golden", "nvfp4_golden.json")) as f:
    NV = json.load(f)


def _sha(t) -> str:
    return hashlib.sha256(t.contiguous().cpu().numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("case", NV["quantize"], ids=lambda c: c["name"])
def test_quantize_bit_exact_vs_reference(case):
    from recant_b200 import quantize_fast
    x = cases.quantize_input(case).cuda()
    fp = quantize_fast(x, case["rht"], False)
    torch.cuda.synchronize()
    assert _sha(fp.codes) == case["codes"]
    assert _sha(fp.scales.view(torch.uint8)) == case["scales"]
    assert _sha(fp.blocked) == case["blocked"]
    assert float(fp.gscale.cpu()).hex() == case["gscale"]


@pytest.mark.parametrize("shape", [(16384, 4096), (4096, 12288), (1000, 4096 + 16)])
def test_quantize_bit_exact_large_vs_oracle(shape):
    gen = torch.Generator().manual_seed(shape[0])
    x = torch.randn(*shape, generator=gen).to(torch.bfloat16)
    from recant_b200 import quantize_fast
    fp = quantize_fast(x.cuda(), True, False)
    c, s, g = ON.quantize_activation(x.float().numpy(), "bf16", True)
    assert np.array_equal(fp.codes.cpu().numpy(), c)
    assert np.array_equal(fp.scales.view(torch.uint8).cpu().numpy(), s)
    assert np.array_equal(fp.blocked.cpu().numpy(), ON.to_blocked(s))
    assert float(fp.gscale.cpu()) == float(g)


def test_stochastic_rounding_unbiased_and_neighbouring():
    """recant/selfcheck.py:22-27: mean of 64 SR draws within 3% of rht(x); every SR code is one of
    the two grid neighbours of the exactly scaled value, and the scales equal the RN scales."""
    from recant_b200 import quantize_fast
    gen = torch.Generator().manual_seed(4)
    x = (torch.randn(64, 256, generator=gen) * 2).to(torch.bfloat16)
    target = ON.rht(x.float().numpy(), "bf16")
    rn_c, rn_s, rn_g = ON.quantize(target)
    acc = np.zeros_like(target)
    xd = x.cuda()
    codes_seen = set()
    for i in range(64):
        fp = quantize_fast(xd, True, True, seed=1000 + i)
        c, s, g = fp.codes.cpu().numpy(), fp.scales.view(torch.uint8).cpu().numpy(), float(fp.gscale.cpu())
        assert np.array_equal(s, rn_s) and g == float(rn_g)
        deq = ON.dequant(c, s, g, 256)
        acc += deq
        codes_seen.add(_sha(fp.codes))
        # neighbour check
        denom = (np.where(ON.e4m3_decode(s) == 0, 1.0, ON.e4m3_decode(s)) * np.float32(g)).astype(np.float32)
        q = target.reshape(64, 16, 16) / denom[..., None]
        a = np.minimum(np.abs(q), 6.0)
        val = np.abs(ON.FP4_GRID[ON.unpack(c, 256) & 7].reshape(64, 16, 16))
        lo = ON.FP4_GRID[np.maximum((a[..., None] > ON.FP4_GRID).sum(-1), 1) - 1]
        hi = ON.FP4_GRID[np.maximum((a[..., None] > ON.FP4_GRID).sum(-1), 1)]
        assert np.all((val == lo) | (val == hi))
    acc /= 64
    assert np.abs(acc - target).mean() / np.abs(target).mean() < 0.03
    assert len(codes_seen) > 1


@pytest.mark.parametrize("shape", [(1, 4096), (3, 48), (8, 4096), (9, 4096), (129, 256)])
@pytest.mark.parametrize("dtype,rht", [("bf16", True), ("bf16", False), ("f32", True)])
def test_quantize_single_launch_and_sweep_paths_bit_exact(shape, dtype, rht):
    """Up to 2048 blocks of 16 take the one-CTA kernel, more take the two sweeps: shapes on both
    sides of the boundary (8 x 4096 = 2048 blocks, 9 x 4096 = 2304), a decode-sized row, and ragged
    ones whose blocked scales have pad rows and columns. Rows of exact rounding midpoints are mixed in
    so that ties take the exact path. The pads must come back zero even over dirty memory."""
    from recant_b200 import quantize_fast
    m, k = shape
    gen = torch.Generator().manual_seed(m * 7 + k)
    x = torch.randn(m, k, generator=gen) * 2
    ties = torch.tensor([6.0, 0.75, 1.75, 3.5, 0.25, 1.25, 2.5, 5.0, -0.75, -1.75, -3.5, -5.0, 0.0, -0.0, 3.0, -6.0])
    x[::2] = ties.repeat(k // 16)[None, :].expand(x[::2].shape) * (1.0 + torch.arange(x[::2].shape[0])[:, None])
    td = torch.bfloat16 if dtype == "bf16" else torch.float32
    x = x.to(td)
    dirty = torch.full((1 << 22,), 255, dtype=torch.uint8, device="cuda")
    del dirty
    fp = quantize_fast(x.cuda(), rht, False)
    c, s, g = ON.quantize_activation(x.float().numpy(), dtype, rht)
    assert np.array_equal(fp.codes.cpu().numpy(), c)
    assert np.array_equal(fp.scales.view(torch.uint8).cpu().numpy(), s)
    assert np.array_equal(fp.blocked.cpu().numpy(), ON.to_blocked(s))
    assert float(fp.gscale.cpu()) == float(g)
