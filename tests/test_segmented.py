"""The affine segment hand-off on the CPU oracle (small head dim): per-segment maps composed with
prefix / suffix folds reproduce the unsegmented op, and the rank-level folds used by context
parallelism agree across a world_size-2 gloo group."""
import os

import torch
import torch.multiprocessing as mp

from oracle import gdn as OG
from oracle import inputs as I
from oracle import segments as SG


def _problem(T=320, d=8, H=2, seed=0):
    inp = I.gdn_inputs(1, T, H, H, d, dtype=torch.float64, seed=seed)
    inp = {k: v.double() for k, v in inp.items()}
    return inp


def _seg_maps(inp, bounds, d, H):
    """Per-segment (M, S0) from the oracle by linearity: S0 = walk(0), M = walk(I) - walk(0)."""
    eye = torch.eye(d, dtype=torch.float64).expand(1, H, d, d)
    Ms, S0 = [], []
    for s, e in zip(bounds[:-1], bounds[1:]):
        args = [inp[n][:, s:e] for n in ("q", "k", "v", "g", "beta")]
        _, z = OG.gdn_forward(*args, torch.zeros(1, H, d, d, dtype=torch.float64), True, dtype=torch.float64)
        _, one = OG.gdn_forward(*args, eye.clone(), True, dtype=torch.float64)
        S0.append(z.double()[0])
        Ms.append((one.double() - z.double())[0])
    return torch.stack(Ms), torch.stack(S0)


def test_prefix_reproduces_unsegmented_forward():
    d, H = 8, 2
    inp = _problem(d=d, H=H)
    bounds = [0, 64, 192, 256, 320]
    Ms, S0 = _seg_maps(inp, bounds, d, H)
    h0 = torch.randn(H, d, d, dtype=torch.float64) * 0.1
    S_in = SG.prefix(Ms, S0, h0)
    o_full, hT_full = OG.gdn_forward(*(inp[n] for n in ("q", "k", "v", "g", "beta")), h0[None], True, dtype=torch.float64)
    for kk, (s, e) in enumerate(zip(bounds[:-1], bounds[1:])):
        o, hT = OG.gdn_forward(*(inp[n][:, s:e] for n in ("q", "k", "v", "g", "beta")), S_in[kk][None], True,
                               dtype=torch.float64)
        assert torch.allclose(o, o_full[:, s:e], atol=1e-5)
    M, c = SG.compose(Ms, S0)
    assert torch.allclose(M @ h0 + c, hT_full[0].double(), atol=1e-5)


def test_suffix_matches_autograd_state_gradient():
    d, H = 8, 2
    inp = _problem(d=d, H=H, seed=2)
    bounds = [0, 128, 192, 320]
    Ms, S0 = _seg_maps(inp, bounds, d, H)
    d_final = torch.randn(H, d, d, dtype=torch.float64)
    # gradient of <S_final, d_final> w.r.t. the initial state through the composed map = M^T d_final
    M, _ = SG.compose(Ms, S0)
    dS_out = SG.suffix(Ms, torch.zeros_like(S0), d_final)
    assert torch.allclose(Ms[0].transpose(-1, -2) @ dS_out[0], M.transpose(-1, -2) @ d_final, atol=1e-8)
    h0 = torch.zeros(1, H, d, d, dtype=torch.float64, requires_grad=True)
    _, hT = OG.gdn_forward(*(inp[n] for n in ("q", "k", "v", "g", "beta")), h0, True, dtype=torch.float64)
    (hT.double() * d_final).sum().backward()
    assert torch.allclose(h0.grad[0], M.transpose(-1, -2) @ d_final, atol=1e-5)


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        d, H = 8, 2
        inp = _problem(d=d, H=H, seed=5)
        shards = [[0, 64, 128], [128, 192, 320]]           # two segments per rank
        Ms, S0 = _seg_maps(inp, shards[rank], d, H)
        Mr, cr = SG.compose(Ms, S0)
        packed = torch.stack([Mr, cr], 0)
        gathered = [torch.empty_like(packed) for _ in range(world)]
        dist.all_gather(gathered, packed)
        M_all = torch.stack([x[0] for x in gathered])
        c_all = torch.stack([x[1] for x in gathered])
        h0 = torch.full((H, d, d), 0.05, dtype=torch.float64)
        s_in = SG.rank_input_state(M_all, c_all, rank, h0)
        S_in = SG.prefix(Ms, S0, s_in)
        outs = []
        for kk, (s, e) in enumerate(zip(shards[rank][:-1], shards[rank][1:])):
            o, _ = OG.gdn_forward(*(inp[n][:, s:e] for n in ("q", "k", "v", "g", "beta")), S_in[kk][None], True,
                                  dtype=torch.float64)
            outs.append(o)
        d_final = torch.full((H, d, d), 0.3, dtype=torch.float64)
        dz = torch.zeros(H, d, d, dtype=torch.float64)
        local = dz
        for kk in range(Ms.shape[0] - 1, -1, -1):
            local = Ms[kk].transpose(-1, -2) @ local
        dg_ = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(dg_, local)
        d_out = SG.rank_output_grad(M_all, torch.stack(dg_), rank, d_final)
        out[rank] = (torch.cat(outs, 1), d_out)
    finally:
        dist.destroy_process_group()


def test_context_parallel_rank_folds_gloo():
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    ctx = mp.get_context("spawn")
    port = 29700 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p_ in procs:
        p_.start()
    for p_ in procs:
        p_.join(120)
        assert p_.exitcode == 0
    d, H = 8, 2
    inp = _problem(d=d, H=H, seed=5)
    h0 = torch.full((1, H, d, d), 0.05, dtype=torch.float64)
    o_full, _ = OG.gdn_forward(*(inp[n] for n in ("q", "k", "v", "g", "beta")), h0, True, dtype=torch.float64)
    assert torch.allclose(out[0][0], o_full[:, :128], atol=1e-5)
    assert torch.allclose(out[1][0], o_full[:, 128:], atol=1e-5)
    # rank 0's outgoing-state gradient = rank 1's map transposed applied to d_final
    Ms1, S01 = _seg_maps(inp, [128, 192, 320], d, H)
    M1, _ = SG.compose(Ms1, S01)
    d_final = torch.full((H, d, d), 0.3, dtype=torch.float64)
    assert torch.allclose(out[0][1], M1.transpose(-1, -2) @ d_final, atol=1e-6)
    assert torch.allclose(out[1][1], d_final)
