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


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
