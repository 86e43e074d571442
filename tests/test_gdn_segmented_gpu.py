"""Segmented GDN (affine state hand-off between chunk-aligned segments walked in parallel) vs the
fp32 oracle over the unsegmented sequence: bf16 inputs, tolerance 2e-2 relative Frobenius; and
vs the unsegmented tensor-core op, which it must track far more closely."""
import os
import subprocess
import sys

import pytest
import torch

from gpu_util import rel
from oracle import gdn as OG
from oracle import inputs as I

pytestmark = pytest.mark.gpu
TOL = 2e-2
NAMES = ("q", "k", "v", "g", "beta")


def _run(fn, inp, do, h0, dht, **kw):
    leaves = {n: inp[n].cuda().detach().clone().requires_grad_(True) for n in NAMES}
    h0d = None if h0 is None else h0.cuda().clone().requires_grad_(True)
    o, hT = fn(*(leaves[n] for n in NAMES), h0d, True, **kw)
    loss = (o.float() * do.cuda().float()).sum()
    if dht is not None:
        loss = loss + (hT * dht.cuda()).sum()
    loss.backward()
    torch.cuda.synchronize()
    gr = {n: leaves[n].grad.cpu() for n in NAMES}
    if h0d is not None:
        gr["h0"] = h0d.grad.cpu()
    return o.detach().cpu(), hT.detach().cpu(), gr


@pytest.mark.parametrize("T,Hk,Hv,seg,with_state", [(1000, 2, 4, 128, True), (1000, 2, 4, 64, False),
                                                     (4096, 4, 4, 1024, True), (300, 1, 2, 1024, True)])
def test_segmented_matches_oracle_and_unsegmented(T, Hk, Hv, seg, with_state):
    from recant_b200 import gdn_b200, gdn_segmented
    inp = I.gdn_inputs(1, T, Hk, Hv, 128, dtype=torch.bfloat16, seed=T + seg)
    gen = torch.Generator().manual_seed(T)
    inp["g"] = -torch.rand(1, T, Hv, generator=gen) * 0.2          # mild decay: the state carries far
    do = I.grad_output(1, T, Hv, 128, dtype=torch.bfloat16, seed=T + 3)
    h0 = torch.randn(1, Hv, 128, 128, generator=gen) * 0.1 if with_state else None
    dht = torch.randn(1, Hv, 128, 128, generator=gen) * 0.1 if with_state else None
    f32 = {n: t.float() for n, t in inp.items()}
    ro, rhT, rg = OG.gdn_fwd_bwd(*(f32[n] for n in NAMES), do.float(), h0, dht)
    so, shT, sg = _run(gdn_segmented, inp, do, h0, dht, segment_len=seg)
    fo, fhT, fg = _run(gdn_b200, inp, do, h0, dht, path="fast")
    errs = {"o": rel(so, ro), "hT": rel(shT, rhT)}
    errs.update({"d" + n: rel(sg[n], rg[n]) for n in NAMES})
    near = {"o": rel(so, fo), "hT": rel(shT, fhT)}
    near.update({"d" + n: rel(sg[n], fg[n]) for n in NAMES})
    if with_state:
        errs["dh0"] = rel(sg["h0"], rg["h0"])
        near["dh0"] = rel(sg["h0"], fg["h0"])
    bad = {k: v for k, v in errs.items() if not v < TOL}
    assert not bad, (bad, errs)
    far = {k: v for k, v in near.items() if not v < 1e-2}
    assert not far, (far, near)


def test_segmented_rejects_unsupported():
    from recant_b200 import gdn_segmented
    x = torch.zeros(2, 64, 1, 128, dtype=torch.bfloat16, device="cuda")
    g = torch.zeros(2, 64, 1, device="cuda")
    with pytest.raises(ValueError):
        gdn_segmented(x, x, x, g, g.bfloat16(), segment_len=128)
    with pytest.raises(ValueError):
        gdn_segmented(x[:1], x[:1], x[:1], g[:1], g[:1].bfloat16(), segment_len=100)


CP_SCRIPT = os.path.join(os.path.dirname(__file__), "cp_worker.py")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="context parallelism needs 2 GPUs")
def test_context_parallel_two_ranks():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(29400 + os.getpid() % 500), CP_SCRIPT]
    res = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "CP OK" in res.stdout, res.stdout[-3000:]


@pytest.mark.parametrize("transpose", [False, True])
@pytest.mark.parametrize("n", [0, 1, 5])
def test_state_fold_kernel_matches_oracle(n, transpose):
    from oracle import segments as OS
    from recant_b200.segmented import state_fold
    gen = torch.Generator().manual_seed(n + 10 * transpose)
    H = 3
    M = torch.randn(n, H, 128, 128, generator=gen) / 128 ** 0.5
    c = torch.randn(n, H, 128, 128, generator=gen)
    s0 = torch.randn(H, 128, 128, generator=gen)
    states, final = state_fold(M.cuda(), c.cuda(), s0.cuda(), transpose=transpose)
    rs, rf = OS.fold(M.double(), c.double(), s0.double(), transpose=transpose)
    assert rel(final, rf) < 1e-5
    if n:
        assert rel(states, rs) < 1e-5
        # identity start without offsets composes the maps
        _, prod = state_fold(M.cuda(), identity=True, states=False, transpose=transpose)
        eye = torch.eye(128, dtype=torch.float64).expand(H, 128, 128)
        assert rel(prod, OS.fold(M.double(), None, eye, transpose=transpose)[1]) < 1e-5


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("n_pre,n", [(0, 4), (3, 4), (2, 0)])
def test_state_fold_modes_and_prefix_run(mode, n_pre, n):
    """rb2_gdn_state_fold_ex: mode 2 (ascending, applying the transpose of the given maps) and a prefix
    run applied first without recording its entering values, against the oracle fold of the
    concatenated maps."""
    from oracle import segments as OS
    from recant_b200.segmented import state_fold
    gen = torch.Generator().manual_seed(31 * mode + 7 * n_pre + n)
    H = 2
    Mp = torch.randn(n_pre, H, 128, 128, generator=gen) / 128 ** 0.5
    cp = torch.randn(n_pre, H, 128, 128, generator=gen)
    M = torch.randn(n, H, 128, 128, generator=gen) / 128 ** 0.5
    c = torch.randn(n, H, 128, 128, generator=gen)
    s0 = torch.randn(H, 128, 128, generator=gen)
    pre = (Mp.cuda(), cp.cuda()) if n_pre else None
    states, final = state_fold(M.cuda(), c.cuda(), s0.cuda(), mode=mode, prefix=pre)
    # the same walk in the oracle: mode 2 applies M^T in forward order
    A = lambda t: t.transpose(-1, -2).contiguous() if mode == 2 else t
    if mode == 1:  # descending: the prefix runs first, i.e. it is the tail of the concatenation
        allM, allc = torch.cat([M, Mp]), torch.cat([c, cp])
        rs, rf = OS.fold(allM.double(), allc.double(), s0.double(), transpose=True)
        ref_states = rs[:n]
    else:
        allM, allc = torch.cat([A(Mp), A(M)]), torch.cat([cp, c])
        rs, rf = OS.fold(allM.double(), allc.double(), s0.double())
        ref_states = rs[n_pre:]
    assert rel(final, rf) < 1e-5
    if n:
        assert rel(states, ref_states) < 1e-5
