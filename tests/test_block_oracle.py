"""The GDN-block oracle (oracle/block.py) against the reference block's own output."""
import torch

from block_util import HK, HV, golden, oracle_params
from oracle import block as OB


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def test_block_oracle_matches_reference_output():
    G = golden()
    P = oracle_params(G)
    with torch.no_grad():
        out = OB.block_forward(G["x"].to(torch.bfloat16), P, HK, HV)
    # same algorithm; matmul summation order (float64 here, float32 in the reference) may flip an
    # occasional bf16 rounding
    assert rel(out.float(), G["out"]) < 5e-3, rel(out.float(), G["out"])


def test_block_oracle_backward_runs_and_reaches_lora():
    G = golden()
    P = oracle_params(G, requires_grad=True)
    x = G["x"][:, :40].to(torch.bfloat16).requires_grad_(True)
    out = OB.block_forward(x, P, HK, HV)
    out.float().pow(2).mean().backward()
    assert x.grad is not None and torch.isfinite(x.grad.float()).all()
    for name in ("in_proj_qkv", "in_proj_z", "out_proj"):
        assert P[name]["A"].grad is not None and P[name]["B"].grad.abs().sum() > 0
