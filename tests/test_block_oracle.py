"""The GDN-block oracle (oracle/block.py) against the reference block's own output."""
import torch

from block_util import HK, HV, golden, oracle_params
from oracle import block as OB


# Oracle vs the reference's outputs: 0 on the machine that generated the fixtures. A different BLAS
# summation order can move a product by an ulp, flip an NVFP4 code next to a decision point and so
# change a short output by up to a few percent; 2e-2 allows that and nothing more.
ORACLE_TOL = 2e-2


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def test_block_oracle_matches_reference_output():
    G = golden()
    P = oracle_params(G)
    with torch.no_grad():
        out = OB.block_forward(G["x"].to(torch.bfloat16), P, HK, HV)
    # bit-identical where the fixture was made (the oracle's emulated GEMM is the reference's own
    # float32 torch call); the bound covers another CPU's sgemm summation order flipping a code
    assert rel(out.float(), G["out"]) < ORACLE_TOL, rel(out.float(), G["out"])


def test_block_oracle_backward_runs_and_reaches_lora():
    G = golden()
    P = oracle_params(G, requires_grad=True)
    x = G["x"][:, :40].to(torch.bfloat16).requires_grad_(True)
    out = OB.block_forward(x, P, HK, HV)
    out.float().pow(2).mean().backward()
    assert x.grad is not None and torch.isfinite(x.grad.float()).all()
    for name in ("in_proj_qkv", "in_proj_z", "out_proj"):
        assert P[name]["A"].grad is not None and P[name]["B"].grad.abs().sum() > 0


def test_block_oracle_decode_matches_reference_cache_path():
    """Prefill, single-token steps and a short chunk through a cache (the serving loop) against the
    reference block's outputs and cache states."""
    from block_util import Cache, decode_golden
    G, D = golden(), decode_golden()
    P = oracle_params(G)
    x = D["x"].to(torch.bfloat16)
    cache = Cache()
    with torch.no_grad():
        for i, (s, e) in enumerate(D["calls"].tolist()):
            out = OB.block_forward(x[:, s:e], P, HK, HV, cache=cache)
            assert rel(out.float(), D[f"out{i}"]) < ORACLE_TOL, (i, rel(out.float(), D[f"out{i}"]))
            assert rel(cache.conv_state.float(), D[f"conv_state{i}"]) < ORACLE_TOL, i
            if f"rec_state{i}" in D:
                assert rel(cache.rec_state, D[f"rec_state{i}"]) < ORACLE_TOL, i
