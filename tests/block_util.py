"""Loading the GDN-block golden fixture (tests/golden/block_golden.npz, made by the reference's
``GatedDeltaNet``; see tests/golden/make_golden.py) for the oracle and the B200 block."""
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
HK, HV, HIDDEN = 1, 2, 256
LORA_SCALE = 32 / 16


def golden():
    z = np.load(os.path.join(HERE, "golden", "block_golden.npz"))
    return {k: torch.from_numpy(z[k]) for k in z.files}


def oracle_params(G, requires_grad=False):
    """Parameters for oracle.block.block_forward (bf16 weights, NVFP4 by oracle.nvfp4)."""
    from oracle import block as OB
    bf = torch.bfloat16
    P = {}
    for name in ("in_proj_qkv", "in_proj_z", "out_proj"):
        A = G[name + ".lora_A"].clone().requires_grad_(requires_grad)
        B = G[name + ".lora_B"].clone().requires_grad_(requires_grad)
        P[name] = OB.quantized(G[name + ".weight"].to(bf), (A, B, LORA_SCALE))
    for name in ("in_proj_b", "in_proj_a"):
        P[name] = {"weight": G[name + ".weight"].to(bf)}
    P["conv"] = G["conv1d.weight"].to(bf)
    P["A_log"], P["dt_bias"] = G["A_log"].to(bf), G["dt_bias"].to(bf)
    P["norm"] = G["norm.weight"].to(bf)
    return P


def decode_golden():
    """tests/golden/block_decode_golden.npz: the reference block with a LayerCache over a prefill,
    three single-token steps and a 5-token chunk (tests/golden/make_golden.py:decode_main)."""
    z = np.load(os.path.join(HERE, "golden", "block_decode_golden.npz"))
    return {k: torch.from_numpy(z[k]) for k in z.files}


class Cache:
    """A LayerCache stand-in: the two fields GatedDeltaNet.forward reads and replaces."""

    def __init__(self):
        self.conv_state = None
        self.rec_state = None
