"""Generate the golden fixtures by running the REFERENCE package on seeded CPU inputs.

Run in a container where the reference RECANT checkout is importable:

    python tests/golden/make_golden.py /path/to/reference

It writes ``tests/golden/nvfp4_golden.json`` (sha256 of codes / scale bytes / blocked scales
and the exact global scale of ``quantize(rht(x))`` for the reference's own self-check cases,
recant/selfcheck.py:9-21, plus weight quantisation and an emulated GEMM) and
``tests/golden/gdn_golden.npz`` (fp32 forward outputs and autograd gradients of
``recant.model.ops.gdn_torch``).  Inputs are regenerated from seeds by the same recipes in
``tests/golden/cases.py``, so only outputs are stored.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

import cases  # noqa: E402


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from recant.model import nvfp4 as R
    from recant.model import ops as RO

    out = {"quantize": [], "weights": [], "gemm": []}
    for case in cases.quantize_cases():
        x = cases.quantize_input(case)
        y = R.rht(x) if case["rht"] else x
        fp = R.quantize(y)
        out["quantize"].append({**case,
                                "codes": sha(fp.codes), "scales": sha(fp.scales.view(torch.uint8)),
                                "blocked": sha(R._to_blocked(fp.scales).view(torch.uint8)),
                                "gscale": float(fp.gscale).hex()})
    for case in cases.weight_cases():
        w = cases.weight_input(case)
        W = R.quantize_weight(w)
        out["weights"].append({**case,
                               "fprop_codes": sha(W.fprop.codes),
                               "fprop_scales": sha(W.fprop.scales.view(torch.uint8)),
                               "fprop_gscale": float(W.fprop.gscale).hex(),
                               "dgrad_codes": sha(W.dgrad.codes),
                               "dgrad_scales": sha(W.dgrad.scales.view(torch.uint8)),
                               "dgrad_gscale": float(W.dgrad.gscale).hex()})
    arrays = {}
    for case in cases.gemm_cases():
        x, w = cases.gemm_input(case)
        a = R.quantize(R.rht(x))
        W = R.quantize_weight(w)
        y = R._gemm_emulated(a, W.fprop)
        arrays[f"gemm_{case['name']}"] = y.numpy()
        out["gemm"].append(case)
    with open(os.path.join(HERE, "nvfp4_golden.json"), "w") as f:
        json.dump(out, f, indent=1)

    for case in cases.gdn_cases():
        inp, do, h0, dht = cases.gdn_input(case)
        hv = inp["v"].shape[2]
        leaves = {n: inp[n].clone().requires_grad_(True) for n in ("q", "k", "v", "g", "beta")}
        h0l = h0.clone().requires_grad_(True) if h0 is not None else None
        # the reference caller repeats q/k heads to Hv before calling the op
        rep = lambda t: t.repeat_interleave(hv // t.shape[2], dim=2) if t.shape[2] != hv else t
        o, hT = RO.gdn_torch(rep(leaves["q"]), rep(leaves["k"]), leaves["v"], leaves["g"],
                             leaves["beta"], h0l, True)
        loss = (o.float() * do.float()).sum() + (hT * dht).sum()
        loss.backward()
        nm = case["name"]
        arrays[f"{nm}_o"] = o.detach().float().numpy()
        arrays[f"{nm}_hT"] = hT.detach().numpy()
        for n, t in leaves.items():
            arrays[f"{nm}_d{n}"] = t.grad.float().numpy()
        if h0l is not None:
            arrays[f"{nm}_dh0"] = h0l.grad.numpy()
    np.savez_compressed(os.path.join(HERE, "golden_arrays.npz"), **arrays)
    print("wrote", sorted(arrays))


def _reference_block(ref_root: str):
    """The reference ``GatedDeltaNet`` (recant/model/layers.py:133-182) at a small bf16
    configuration (hidden 256, Hk 1, Hv 2, head dim 128) with NVFP4 projections and rank-16 LoRA
    (random B so that LoRA contributes), and its weights (fp32 values of the bf16 parameters, taken
    before quantisation). Returns (block, arrays, generator, layers module)."""
    sys.path.insert(0, ref_root)
    from recant.model import layers
    from recant.model.config import TextConfig
    c = TextConfig(hidden_size=256, linear_key_head_dim=128, linear_value_head_dim=128, linear_num_key_heads=1,
                   linear_num_value_heads=2, num_hidden_layers=1)
    torch.manual_seed(11)
    gen = torch.Generator().manual_seed(11)
    blk = layers.GatedDeltaNet(c)
    with torch.no_grad():
        for name in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj"):
            lin = getattr(blk, name)
            lin.weight.copy_(torch.randn(lin.weight.shape, generator=gen) * 0.06)
        blk.conv1d.weight.copy_(torch.randn(blk.conv1d.weight.shape, generator=gen) * 0.4)
        blk.A_log.copy_(torch.log(torch.empty(2).uniform_(1.0, 16.0, generator=gen)))
        blk.dt_bias.copy_(torch.randn(2, generator=gen) * 0.5)
        blk.norm.weight.copy_(1.0 + 0.1 * torch.randn(128, generator=gen))
    blk = blk.to(torch.bfloat16)
    arrays = {}
    for name, prm in blk.named_parameters():
        arrays[name] = prm.detach().float().numpy()
    for name in ("in_proj_qkv", "in_proj_z", "out_proj"):
        lin = getattr(blk, name)
        lin.quantize_(True)
        lin.add_lora(16, 32)
        with torch.no_grad():
            lin.lora_B.copy_(torch.randn(lin.lora_B.shape, generator=gen) * 0.02)
        arrays[name + ".lora_A"] = lin.lora_A.detach().numpy()
        arrays[name + ".lora_B"] = lin.lora_B.detach().numpy()
    return blk, arrays, gen, layers


def block_main(ref_root: str) -> None:
    """``tests/golden/block_golden.npz``: the reference block's weights, a seeded input [1, 70, 256],
    the forward output and out_proj's input ``y`` (the gated norm's output, before out_proj quantizes
    it to NVFP4), captured by a forward pre-hook on the reference's out_proj."""
    blk, arrays, gen, _ = _reference_block(ref_root)
    x = torch.randn(1, 70, 256, generator=gen).to(torch.bfloat16)
    seen = {}
    hook = blk.out_proj.register_forward_pre_hook(lambda mod, args: seen.setdefault("y", args[0].detach().clone()))
    with torch.no_grad():
        out = blk(x)
    hook.remove()
    arrays["x"] = x.float().numpy()
    arrays["out"] = out.float().numpy()
    arrays["y"] = seen["y"].float().numpy()
    np.savez_compressed(os.path.join(HERE, "block_golden.npz"), **arrays)
    print("block golden: out", tuple(out.shape), float(out.float().abs().mean()))


def decode_main(ref_root: str) -> None:
    """``tests/golden/block_decode_golden.npz``: the same reference block (weights in
    block_golden.npz) driven as the serving engine drives it (serve/engine.py:107-119), with a
    ``LayerCache`` (layers.py:111-130) over 2 sequences of a seeded input [2, 48, 256]: a 40-token
    prefill, three single-token steps, then a 5-token chunk. Stores every output, out_proj's input
    ``y`` of every call (forward pre-hook), the cache's conv state after each call and its
    recurrent state after the prefill and at the end."""
    blk, _, _, layers = _reference_block(ref_root)
    gen = torch.Generator().manual_seed(12)
    x = torch.randn(2, 48, 256, generator=gen).to(torch.bfloat16)
    cache = layers.LayerCache()
    calls = [(0, 40), (40, 41), (41, 42), (42, 43), (43, 48)]
    arrays = {"x": x.float().numpy()}
    seen = []
    hook = blk.out_proj.register_forward_pre_hook(lambda mod, args: seen.append(args[0].detach().clone()))
    with torch.no_grad():
        for i, (s, e) in enumerate(calls):
            out = blk(x[:, s:e], cache, s)
            arrays[f"out{i}"] = out.float().numpy()
            arrays[f"y{i}"] = seen[-1].float().numpy()
            arrays[f"conv_state{i}"] = cache.conv_state.float().numpy()
            if i in (0, len(calls) - 1):  # after the prefill and at the end
                arrays[f"rec_state{i}"] = cache.rec_state.float().numpy()
    hook.remove()
    arrays["calls"] = np.array(calls, dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "block_decode_golden.npz"), **arrays)
    print("decode golden:", [tuple(arrays[f"out{i}"].shape) for i in range(len(calls))])


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path of the reference RECANT checkout>")
    root = sys.argv[1]
    main(root)
    block_main(root)
    decode_main(root)
