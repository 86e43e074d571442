"""Host-side choices of the GDN block's LoRA paths (CPU): which products take this library's LoRA
kernels and when a scale can be folded into a product exactly."""
import torch

import recant_b200.block as blk


def test_pow2_scales_fold_exactly():
    """alpha / r is folded into the backward's products only when scaling by it is exact."""
    assert all(blk._pow2(s) for s in (1.0, 2.0, 0.5, 4.0, 0.125))
    assert not any(blk._pow2(s) for s in (3.0, 0.3, 1.5, 0.0, -2.0))
    # and it is exact: a power-of-two scale commutes with bf16 rounding of any product
    g = torch.Generator().manual_seed(0)
    a = torch.randn(1000, generator=g)
    for s in (2.0, 0.5):
        assert torch.equal((a * s).to(torch.bfloat16), a.to(torch.bfloat16) * s)


def test_lora_kernels_refuse_cpu_tensors_and_follow_their_switches(monkeypatch):
    """CPU tensors keep the reference's torch ops, decode-sized products are below the up-projection
    kernel's row threshold, and the switches turn the LoRA kernels off."""
    y = torch.zeros(128, 256, dtype=torch.bfloat16)
    h = torch.zeros(128, 16, dtype=torch.bfloat16)
    b = torch.zeros(256, 16, dtype=torch.bfloat16)
    assert not blk._use_up(y, h, b)                # CPU tensors
    assert not blk._wgrad_ok(y, h)
    assert not blk._lora_kernels_ok(y)
    assert blk.LORA_UP_MIN_ROWS > 4                # decode-sized products stay on the torch ops
    monkeypatch.setattr(blk, "LORA_UP", False)
    monkeypatch.setattr(blk, "LORA_WGRAD", False)
    assert not blk._lora_kernels_ok(y)
