"""Data-parallel host logic on CPU: LPT balance, local packs, and a world_size-2 gloo run whose
per-rank results (CPU oracle GDN per rank + all-reduced bucket) equal the single-process ones."""
import os

import pytest
import torch
import torch.multiprocessing as mp

from oracle import gdn as OG
from oracle import inputs as I
from recant_b200 import parallel as P


def test_config3_lengths_and_balance():
    lengths = I.varlen_lengths()
    assert len(lengths) == 64 and sum(lengths) == 243613
    for world in (1, 2, 4, 8):
        parts, loads = P.lpt_partition(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(64))
        assert sum(loads) == sum(lengths)
        # LPT bound: max load <= mean + longest sequence
        assert max(loads) <= sum(lengths) / world + max(lengths)
        if world > 1:
            assert max(loads) / (sum(lengths) / world) < 1.05
    # deterministic
    assert P.lpt_partition(lengths, 8) == P.lpt_partition(lengths, 8)


def test_lora_bucket_size_matches_config3():
    assert P.lora_bucket_numel() == 11_010_048  # 44.0 MB of fp32


def test_local_pack_roundtrip():
    lengths = [5, 9, 1, 7]
    cu = P.cu_seqlens_of(lengths)
    x = torch.arange(sum(lengths)).reshape(1, -1, 1).float()
    (loc,), lcu, spans = P.local_pack([x], cu, [3, 1])
    assert lcu.tolist() == [0, 7, 16]
    assert loc.flatten().tolist() == list(range(15, 22)) + list(range(5, 14))


def _rank_main(rank, world, port, lengths, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        T = sum(lengths)
        inp = I.gdn_inputs(1, T, 1, 2, 128, dtype=torch.float32, seed=3)
        do = I.grad_output(1, T, 2, 128, dtype=torch.float32, seed=4)
        cu = P.cu_seqlens_of(lengths)
        parts, _ = P.lpt_partition(lengths, world)
        names = ("q", "k", "v", "g", "beta")
        loc, lcu, spans = P.local_pack([inp[n] for n in names] + [do], cu, parts[rank])
        o, _, gr = OG.gdn_fwd_bwd(*loc[:5], loc[5], cu_seqlens=lcu)
        bucket = torch.full((1000,), float(rank + 1)) * gr["v"].abs().sum()
        step = P.DataParallelStep()
        step.reduce(bucket)
        out[rank] = (o, gr["v"], spans, bucket)
    finally:
        dist.destroy_process_group()


def test_gloo_dp_matches_single_process():
    lengths = [70, 130, 64, 1, 200, 33]
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    ctx = mp.get_context("spawn")
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, lengths, out)) for r in range(world)]
    for p_ in procs:
        p_.start()
    for p_ in procs:
        p_.join(120)
        assert p_.exitcode == 0
    T = sum(lengths)
    inp = I.gdn_inputs(1, T, 1, 2, 128, dtype=torch.float32, seed=3)
    do = I.grad_output(1, T, 2, 128, dtype=torch.float32, seed=4)
    o_ref, _, gr_ref = OG.gdn_fwd_bwd(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], do,
                                      cu_seqlens=P.cu_seqlens_of(lengths))
    total = 0.0
    for r in range(world):
        o, dv, spans, bucket = out[r]
        off = 0
        for s, e in spans:
            assert torch.allclose(o[:, off:off + e - s], o_ref[:, s:e], atol=1e-6)
            assert torch.allclose(dv[:, off:off + e - s], gr_ref["v"][:, s:e], atol=1e-6)
            off += e - s
        total += (r + 1) * dv.abs().sum().item()
    for r in range(world):
        assert torch.allclose(out[r][3], torch.full((1000,), total), rtol=1e-6)
