"""The GDN block on B200 (recant_b200.block) against the reference's eager CPU ops stage by stage
and against the reference block (golden output) / the block oracle (gradients) end to end."""
import pytest
import torch
import torch.nn.functional as F

from block_util import HIDDEN, HK, HV, golden, oracle_params
from gpu_util import rel
from oracle import block as OB

pytestmark = pytest.mark.gpu


def test_conv_silu_split_forward_backward():
    from recant_b200.block import conv_silu
    gen = torch.Generator().manual_seed(3)
    B, T, C, s1, s2 = 2, 100, 512, 128, 256
    x = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
    w = (torch.randn(C, 1, 4, generator=gen) * 0.4).to(torch.bfloat16)
    dy = torch.randn(B, T, C, generator=gen).to(torch.bfloat16)
    # reference eager path (layers.py:162-166) with autograd on the CPU
    xr = x.clone().requires_grad_(True)
    cat = torch.cat([torch.zeros(B, C, 3, dtype=torch.bfloat16), xr.transpose(1, 2)], -1)
    ref = F.silu(F.conv1d(cat, w, groups=C)).transpose(1, 2)
    ref.backward(dy)
    xd = x.cuda().requires_grad_(True)
    q, k, v = conv_silu(xd, w.cuda(), s1, s2)
    out = torch.cat([q, k, v], -1)
    out.backward(dy.cuda())
    torch.cuda.synchronize()
    assert rel(out.float(), ref.float()) < 1e-2
    assert rel(xd.grad.float(), xr.grad.float()) < 1e-2


def test_gates_forward_backward():
    from recant_b200.block import gdn_gates
    gen = torch.Generator().manual_seed(4)
    a = (torch.randn(3, 50, 8, generator=gen) * 4).to(torch.bfloat16)
    b = torch.randn(3, 50, 8, generator=gen).to(torch.bfloat16)
    A_log = torch.log(torch.empty(8).uniform_(1, 16, generator=gen))
    dt_bias = torch.randn(8, generator=gen)
    dg, db = torch.randn(3, 50, 8, generator=gen), torch.randn(3, 50, 8, generator=gen).to(torch.bfloat16)
    ar, br = a.clone().requires_grad_(True), b.clone().requires_grad_(True)
    g_ref = -A_log.exp() * F.softplus(ar.float() + dt_bias)      # fused_ops.py:32-33
    beta_ref = br.sigmoid()
    (g_ref * dg).sum().backward(retain_graph=True)
    beta_ref.backward(db)
    ad, bd = a.cuda().requires_grad_(True), b.cuda().requires_grad_(True)
    g, beta = gdn_gates(ad, bd, A_log.cuda(), dt_bias.cuda())
    (g * dg.cuda()).sum().backward(retain_graph=True)
    beta.backward(db.cuda())
    assert rel(g, g_ref) < 1e-5 and rel(beta.float(), beta_ref.float()) < 1e-2
    assert rel(ad.grad.float(), ar.grad.float()) < 1e-2 and rel(bd.grad.float(), br.grad.float()) < 1e-2


def test_gated_rmsnorm_forward_backward():
    from recant_b200.block import gated_rmsnorm
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(300, 128, generator=gen).to(torch.bfloat16)
    z = torch.randn(300, 128, generator=gen).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(128, generator=gen)).to(torch.bfloat16)
    dy = torch.randn(300, 128, generator=gen).to(torch.bfloat16)
    xr, zr = x.clone().requires_grad_(True), z.clone().requires_grad_(True)
    y = xr.float()
    y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + 1e-6)   # fused_ops.py:11-16
    y = w * y.to(torch.bfloat16)
    ref = (y * F.silu(zr.float())).to(torch.bfloat16)
    ref.backward(dy)
    xd, zd = x.cuda().requires_grad_(True), z.cuda().requires_grad_(True)
    out = gated_rmsnorm(xd, zd, w.cuda().float())
    out.backward(dy.cuda())
    assert rel(out.float(), ref.float()) < 1e-2
    assert rel(xd.grad.float(), xr.grad.float()) < 2e-2 and rel(zd.grad.float(), zr.grad.float()) < 2e-2


def _block():
    from recant_b200.block import GDNBlock
    G = golden()
    sd = {k: v for k, v in G.items() if k not in ("x", "out")}
    return G, GDNBlock.from_state(sd, HIDDEN, HK, HV)


# The block amplifies rounding differences: re-running the reference's own block with its LoRA
# products as separate ops instead of one addmm moves the output by 3 % (relative Frobenius), so
# end-to-end comparisons use 5e-2; the stages above are compared tightly.
BLOCK_TOL = 5e-2


def test_block_forward_matches_reference_output():
    G, blk = _block()
    with torch.no_grad():
        out = blk(G["x"].to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    assert rel(out.float(), G["out"]) < BLOCK_TOL, rel(out.float(), G["out"])


def test_block_backward_matches_oracle():
    G, blk = _block()
    blk.set_stochastic_backward(False)   # the oracle quantizes dy round-to-nearest
    P = oracle_params(G, requires_grad=True)
    x = G["x"].to(torch.bfloat16)
    gen = torch.Generator().manual_seed(9)
    dy = torch.randn(x.shape, generator=gen).to(torch.bfloat16)
    xr = x.clone().requires_grad_(True)
    OB.block_forward(xr, P, HK, HV).backward(dy)
    xd = x.cuda().requires_grad_(True)
    blk(xd).backward(dy.cuda())
    torch.cuda.synchronize()
    errs = {"dx": rel(xd.grad.float(), xr.grad.float())}
    for name in ("in_proj_qkv", "in_proj_z", "out_proj"):
        lin = getattr(blk, name)
        errs[name + ".A"] = rel(lin.lora_A.grad, P[name]["A"].grad)
        errs[name + ".B"] = rel(lin.lora_B.grad, P[name]["B"].grad)
    # dx goes through the in_proj dgrad GEMMs, which re-quantize dqkv / dz to NVFP4: upstream
    # gradients that differ by ~1e-2 (the LoRA-gradient errors) flip the codes of elements next to a
    # decision point, one e2m1 step each, so dx is compared at 1e-1
    tol = {k: (1e-1 if k == "dx" else BLOCK_TOL) for k in errs}
    bad = {k: v for k, v in errs.items() if not v < tol[k]}
    assert not bad, (bad, errs)


def test_block_stochastic_backward_is_unbiased_around_rn():
    """The default (reference) backward rounds dy stochastically: its input gradient scatters around
    the round-to-nearest one."""
    G, blk = _block()
    x = G["x"].to(torch.bfloat16).cuda()
    dy = torch.randn(x.shape, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).cuda()
    grads = []
    for sr in (False, True, True):
        blk.set_stochastic_backward(sr)
        xd = x.clone().requires_grad_(True)
        blk(xd).backward(dy)
        grads.append(xd.grad.float())
    assert rel(grads[1], grads[0]) < 0.3 and rel(grads[1], grads[2]) > 0
