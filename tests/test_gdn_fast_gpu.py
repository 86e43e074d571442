"""Tensor-core (tcgen05) GDN path vs the fp32 oracle: bf16 inputs, tolerance 2e-2 relative Frobenius."""
import pytest
import torch

from gpu_util import rel
from oracle import gdn as OG
from oracle import inputs as I

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _fwd(inp, h0=None, cu=None):
    from recant_b200 import gdn_b200
    d = {n: t.cuda() for n, t in inp.items()}
    with torch.no_grad():
        o, hT = gdn_b200(d["q"], d["k"], d["v"], d["g"], d["beta"], None if h0 is None else h0.cuda(), True,
                         cu_seqlens=None if cu is None else cu.cuda(), path="fast")
    torch.cuda.synchronize()
    return o.cpu(), hT.cpu()


@pytest.mark.parametrize("B,T,Hk,Hv", [(1, 64, 1, 1), (2, 300, 2, 4), (1, 1024, 4, 8)])
def test_fast_forward(B, T, Hk, Hv):
    inp = I.gdn_inputs(B, T, Hk, Hv, 128, dtype=torch.bfloat16, seed=T + Hv)
    f32 = {n: t.float() for n, t in inp.items()}
    ro, rhT = OG.gdn(f32["q"], f32["k"], f32["v"], f32["g"], f32["beta"], None, True)
    o, hT = _fwd(inp)
    assert rel(o, ro) < TOL and rel(hT, rhT) < TOL, (rel(o, ro), rel(hT, rhT))


def test_fast_forward_initial_state_and_mild_gates():
    inp = I.gdn_inputs(2, 200, 2, 2, 128, dtype=torch.bfloat16, seed=3)
    gen = torch.Generator().manual_seed(3)
    inp["g"] = -torch.rand(2, 200, 2, generator=gen) * 0.1
    h0 = torch.randn(2, 2, 128, 128, generator=gen) * 0.1
    f32 = {n: t.float() for n, t in inp.items()}
    ro, rhT = OG.gdn(f32["q"], f32["k"], f32["v"], f32["g"], f32["beta"], h0, True)
    o, hT = _fwd(inp, h0)
    assert rel(o, ro) < TOL and rel(hT, rhT) < TOL, (rel(o, ro), rel(hT, rhT))


def test_fast_forward_varlen():
    lengths = [70, 1, 64, 0, 129, 33]
    cu = I.cu_seqlens_of(lengths)
    inp = I.gdn_inputs(1, int(cu[-1]), 2, 4, 128, dtype=torch.bfloat16, seed=5)
    f32 = {n: t.float() for n, t in inp.items()}
    ro, rhT = OG.gdn(f32["q"], f32["k"], f32["v"], f32["g"], f32["beta"], None, True, cu_seqlens=cu)
    o, hT = _fwd(inp, cu=cu)
    assert rel(o, ro) < TOL and rel(hT, rhT) < TOL, (rel(o, ro), rel(hT, rhT))


def _check_grads(inp, do, h0=None, dht=None, cu=None):
    from gpu_util import run_b200
    f32 = {n: t.float() for n, t in inp.items()}
    ro, rhT, rg = OG.gdn_fwd_bwd(f32["q"], f32["k"], f32["v"], f32["g"], f32["beta"], do.float(), h0, dht,
                                 cu_seqlens=cu)
    o, hT, gr = run_b200(inp, do, h0, dht, cu=cu, path="fast")
    errs = {"o": rel(o, ro), "hT": rel(hT, rhT)}
    errs.update({"d" + n: rel(gr[n], rg[n]) for n in ("q", "k", "v", "g", "beta")})
    if h0 is not None:
        errs["dh0"] = rel(gr["h0"], rg["h0"])
    bad = {k: v for k, v in errs.items() if not v < TOL}
    assert not bad, (bad, errs)


@pytest.mark.parametrize("B,T,Hk,Hv", [(1, 64, 1, 1), (2, 300, 2, 4), (1, 1024, 4, 8), (2, 130, 2, 2),
                                       (1, 200, 2, 8), (1, 150, 1, 8), (1, 100, 1, 16)])
def test_fast_backward(B, T, Hk, Hv):
    """Includes GQA groups of 2, 4, 8 and 16 value heads per key head."""
    inp = I.gdn_inputs(B, T, Hk, Hv, 128, dtype=torch.bfloat16, seed=T + 7 * Hv)
    do = I.grad_output(B, T, Hv, 128, dtype=torch.bfloat16, seed=T + 1)
    _check_grads(inp, do)


def test_fast_backward_state_grads_and_mild_gates():
    inp = I.gdn_inputs(2, 200, 2, 2, 128, dtype=torch.bfloat16, seed=13)
    gen = torch.Generator().manual_seed(13)
    inp["g"] = -torch.rand(2, 200, 2, generator=gen) * 0.1
    do = I.grad_output(2, 200, 2, 128, dtype=torch.bfloat16, seed=14)
    h0 = torch.randn(2, 2, 128, 128, generator=gen) * 0.1
    dht = torch.randn(2, 2, 128, 128, generator=gen) * 0.1
    _check_grads(inp, do, h0, dht)


def test_fast_backward_varlen():
    lengths = [70, 1, 64, 0, 129, 33]
    cu = I.cu_seqlens_of(lengths)
    T = int(cu[-1])
    inp = I.gdn_inputs(1, T, 2, 4, 128, dtype=torch.bfloat16, seed=21)
    do = I.grad_output(1, T, 4, 128, dtype=torch.bfloat16, seed=22)
    gen = torch.Generator().manual_seed(23)
    h0 = torch.randn(len(lengths), 4, 128, 128, generator=gen) * 0.1
    dht = torch.randn(len(lengths), 4, 128, 128, generator=gen) * 0.1
    _check_grads(inp, do, h0, dht, cu)


def test_outputs_fully_written_over_nan_poisoned_memory():
    """Every element of o, the final state and all input gradients is written by the kernels: the
    caching allocator's free blocks (small and large pools) are filled with NaN before the op runs,
    so anything the kernels leave unwritten or read uninitialised shows up as non-finite. Ragged
    last chunk (T = 130), GQA, an initial state that needs a gradient."""
    from recant_b200 import gdn_b200
    poison = [torch.full((n,), float("nan"), device="cuda") for n in [1 << 26] + [1 << 17] * 64 + [1 << 14] * 64]
    del poison
    inp = I.gdn_inputs(2, 130, 2, 4, 128, dtype=torch.bfloat16, seed=77)
    leaves = {n: t.cuda().requires_grad_(True) for n, t in inp.items()}
    h0 = (torch.randn(2, 4, 128, 128, generator=torch.Generator().manual_seed(78)) * 0.1).cuda().requires_grad_(True)
    o, hT = gdn_b200(leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["beta"], h0, True, path="fast")
    do = torch.randn(o.shape, generator=torch.Generator().manual_seed(79)).to(o.dtype).cuda()
    dhT = torch.randn(hT.shape, generator=torch.Generator().manual_seed(80)).cuda() * 0.1
    torch.autograd.backward([o, hT], [do, dhT])
    torch.cuda.synchronize()
    outs = {"o": o, "hT": hT, "dh0": h0.grad, **{"d" + n: t.grad for n, t in leaves.items()}}
    for name, t in outs.items():
        assert t is not None and bool(torch.isfinite(t.float()).all()), name


def test_fast_headline_shape_parity():
    """One batch row of the benchmark's headline shape: T = 4096 (64 chunks walked per sequence),
    Hk = 16, Hv = 32 (GQA group 2), bf16 inputs from the benchmark's seeded distributions, forward
    and backward against the fp32 oracle. The per-chunk bf16 roundings of the state and of the chunk
    operands compound along the 64-chunk walk; every output and gradient must stay within 2e-2."""
    inp = I.gdn_inputs(1, 4096, 16, 32, 128, dtype=torch.bfloat16, seed=0)
    do = I.grad_output(1, 4096, 32, 128, dtype=torch.bfloat16, seed=1)
    from gpu_util import run_b200
    f32 = {n: t.float() for n, t in inp.items()}
    ro, rhT, rg = OG.gdn_fwd_bwd(f32["q"], f32["k"], f32["v"], f32["g"], f32["beta"], do.float())
    o, hT, gr = run_b200(inp, do, path="fast")
    errs = {"o": rel(o, ro), "hT": rel(hT, rhT)}
    errs.update({"d" + n: rel(gr[n], rg[n]) for n in ("q", "k", "v", "g", "beta")})
    print("headline-shape errors", {k: f"{v:.2e}" for k, v in errs.items()})
    bad = {k: v for k, v in errs.items() if not v < TOL}
    assert not bad, (bad, errs)
