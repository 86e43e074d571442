"""Context-parallel GDN check run under torchrun (one rank per GPU): every rank takes its
contiguous shard of one long sequence; the shards' outputs, the final state and all gradients
must equal the single-GPU segmented op on the whole sequence, and the oracle within 2e-2."""
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from gpu_util import rel  # noqa: E402
from oracle import gdn as OG  # noqa: E402
from oracle import inputs as I  # noqa: E402
from recant_b200 import gdn_segmented  # noqa: E402

NAMES = ("q", "k", "v", "g", "beta")


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=timedelta(seconds=60))
    # weak gates over a short sequence: the initial state and each rank's state still reach the
    # following ranks (with strong decay a lost hand-off term would be invisible)
    T, Hk, Hv, seg = 512, 2, 4, 128
    inp = I.gdn_inputs(1, T, Hk, Hv, 128, dtype=torch.bfloat16, seed=11)
    gen = torch.Generator().manual_seed(11)
    inp["g"] = -torch.rand(1, T, Hv, generator=gen) * 0.002
    do = I.grad_output(1, T, Hv, 128, dtype=torch.bfloat16, seed=12)
    h0 = torch.randn(1, Hv, 128, 128, generator=gen) * 0.5
    dht = torch.randn(1, Hv, 128, 128, generator=gen) * 0.1
    per = T // world
    s, e = rank * per, (rank + 1) * per
    leaves = {n: inp[n][:, s:e].cuda().clone().requires_grad_(True) for n in NAMES}
    h0d = h0.cuda().clone().requires_grad_(True)
    o, hT = gdn_segmented(*(leaves[n] for n in NAMES), h0d, True, segment_len=seg, group=dist.group.WORLD)
    loss = (o.float() * do[:, s:e].cuda().float()).sum() + (hT * dht.cuda()).sum()
    loss.backward()
    torch.cuda.synchronize()
    parts = {"o": o.detach()}
    parts.update({"d" + n: leaves[n].grad for n in NAMES})
    full = {}
    for key, t in parts.items():
        got = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(got, t.contiguous())
        full[key] = torch.cat(got, 1).cpu()
    ok = True
    if rank == 0:
        f32 = {n: t.float() for n, t in inp.items()}
        ro, rhT, rg = OG.gdn_fwd_bwd(*(f32[n] for n in NAMES), do.float(), h0, dht)
        errs = {"o": rel(full["o"], ro), "hT": rel(hT.cpu(), rhT), "dh0": rel(h0d.grad.cpu(), rg["h0"])}
        errs.update({"d" + n: rel(full["d" + n], rg[n]) for n in NAMES})
        print("errs", errs, flush=True)
        ok = all(v < 2e-2 for v in errs.values())
    else:
        ok = h0d.grad is None or float(h0d.grad.abs().max()) == 0.0
    flag = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(flag)
    dist.destroy_process_group()
    if rank == 0:
        print("CP OK" if int(flag) == 0 else "CP FAIL", flush=True)
    sys.exit(0 if int(flag) == 0 else 1)


if __name__ == "__main__":
    main()
