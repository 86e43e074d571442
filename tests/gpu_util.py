"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch


def rel(a, b) -> float:
    a = torch.as_tensor(a).detach().double().cpu()
    b = torch.as_tensor(b).detach().double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def run_b200(inp, do, h0=None, dht=None, cu=None, path="auto", dev="cuda"):
    """Forward + backward through recant_b200.gdn_b200; returns o, hT, grads (on CPU)."""
    from recant_b200 import gdn_b200
    leaves = {n: inp[n].to(dev).detach().clone().requires_grad_(True) for n in ("q", "k", "v", "g", "beta")}
    h0d = None if h0 is None else h0.to(dev).clone().requires_grad_(True)
    cud = None if cu is None else cu.to(dev)
    o, hT = gdn_b200(leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["beta"], h0d, True,
                     cu_seqlens=cud, path=path)
    loss = (o.float() * do.to(dev).float()).sum()
    loss = loss + ((hT * dht.to(dev)).sum() if dht is not None else 0.0 * hT.sum())
    loss.backward()
    grads = {n: t.grad.cpu() for n, t in leaves.items()}
    if h0d is not None:
        grads["h0"] = h0d.grad.cpu()
    torch.cuda.synchronize()
    return o.detach().cpu(), hT.detach().cpu(), grads
