"""Multi-GPU plumbing for the GDN path: data parallelism over packed variable-length sequences.

The reference trains on one GPU (it has no distributed code). Config 3 of the benchmark spec
packs 64 sequences (lengths uniform in [128, 8192]) with ``cu_seqlens`` and splits them across
ranks by token count; each rank runs the varlen GDN forward + backward on its own sequences (no
exchange inside the op: sequences are independent), and the only collective is an NCCL
all-reduce of the LoRA-gradient bucket (24 GDN layers x (qkv, z, out) rank-16 adapters,
11.01 M fp32 = 44 MB) that the surrounding layers produce.

* :func:`lpt_partition` -- longest-processing-time-first assignment of sequences to ranks.
* :func:`local_pack` -- a rank's contiguous token pack and its local ``cu_seqlens``.
* :func:`lora_bucket_numel` -- the bucket size of config 3.
* :class:`DataParallelStep` -- one DP step: local varlen GDN fwd+bwd, then the bucket
  all-reduce (sum) on the process group.
"""
from __future__ import annotations

import heapq

import torch


def lpt_partition(lengths, world: int):
    """Assign sequence indices to ``world`` ranks, longest first onto the least-loaded rank
    (ties: lower rank, then lower index). Returns (per-rank sorted index lists, per-rank tokens)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, r) for r in range(world)]
    parts = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    loads = [sum(int(lengths[i]) for i in p) for p in parts]
    return [sorted(p) for p in parts], loads


def cu_seqlens_of(lengths, device=None):
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + int(n))
    return torch.tensor(cu, dtype=torch.int64, device=device)


def local_pack(tensors, cu_seqlens_global, indices):
    """Gather the token ranges of ``indices`` (in order) from [1, T, ...] tensors into a
    contiguous local pack; returns (local tensors, local cu_seqlens, list of (start, end))."""
    cu = [int(x) for x in cu_seqlens_global]
    spans = [(cu[i], cu[i + 1]) for i in indices]
    out = []
    for t in tensors:
        parts = [t[:, s:e] for s, e in spans]
        out.append(torch.cat(parts, 1) if parts else t[:, :0])
    lens = [e - s for s, e in spans]
    dev = tensors[0].device if tensors else None
    return out, cu_seqlens_of(lens, device=dev), spans


def lora_bucket_numel(layers: int = 24, hidden: int = 4096, rank: int = 16, qkv_out: int = 8192,
                      z_out: int = 4096, out_out: int = 4096) -> int:
    """LoRA parameters (A [r, in], B [out, r]) of in_proj_qkv, in_proj_z and out_proj per layer."""
    per_layer = rank * (hidden + qkv_out) + rank * (hidden + z_out) + rank * (hidden + out_out)
    return layers * per_layer


class DataParallelStep:
    """One data-parallel step of the GDN path on this rank.

    ``forward_backward(inputs, d_o)`` runs ``gdn_b200`` over the rank's pack (B == 1 with local
    ``cu_seqlens``) and backpropagates ``d_o``; ``reduce(bucket)`` all-reduces (sums) the
    gradient bucket in place with the default process group. The bucket is flat fp32 and stays
    allocated across steps.
    """

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group

    def forward_backward(self, inputs, d_o, cu_seqlens, path="auto"):
        from .gdn import gdn_b200
        leaves = {n: t.detach().requires_grad_(True) for n, t in inputs.items()}
        o, _ = gdn_b200(leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["beta"], cu_seqlens=cu_seqlens,
                        path=path)
        o.backward(d_o)
        return o, {n: t.grad for n, t in leaves.items()}

    def reduce(self, bucket: torch.Tensor) -> torch.Tensor:
        if self.dist.is_available() and self.dist.is_initialized() and self.dist.get_world_size() > 1:
            self.dist.all_reduce(bucket, op=self.dist.ReduceOp.SUM, group=self.group)
        return bucket
