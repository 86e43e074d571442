"""rb2_lora_wgrad (the LoRA factor gradients on tcgen05) against a float64 reduction of the same bf16
operands, rounded as the reference's autograd rounds them (the bf16 product, the bf16 multiply by
alpha, the fp32 cast): equal up to one bf16 rounding step where the fp32 sums land next to a
rounding boundary -- relative Frobenius error below 1e-3 and every element within 2^-7 of its
reference plus 2^-12 of the RMS (the fp32 accumulation error of elements that cancel to near
zero). The block-level test runs the GDN block's backward with the kernel and with torch's cuBLAS
products (the reference's own ops) on the same inputs and compares every LoRA gradient."""
import pytest
import torch

from gpu_util import rel

pytestmark = pytest.mark.gpu


def _reference(d, h, scale):
    acc = (d.double().t() @ h.double()).float()           # [N, R], exact to fp32 rounding
    return (acc.to(torch.bfloat16) * scale).to(torch.bfloat16).float() if scale != 1 else acc.to(torch.bfloat16).float()


def _check(out, ref):
    assert rel(out, ref) < 1e-3
    # one bf16 step of each element, plus the fp32 accumulation error of the tensor core's sums over
    # thousands of tokens, which matters for elements that cancel to near zero (2^-12 of the RMS)
    rms = float(ref.double().pow(2).mean().sqrt())
    assert bool(((out - ref).abs() <= ref.abs() * 2.0 ** -7 + rms * 2.0 ** -12).all())


@pytest.mark.parametrize("M,N,R,scale", [(16384, 256, 16, 2.0), (1000, 200, 32, 1.0), (64, 128, 1, 0.5),
                                         (4097, 4096, 64, 2.0), (77, 8, 16, 1.0), (300, 384, 48, 3.0)])
def test_lora_wgrad_matches_float64(M, N, R, scale):
    from recant_b200.block import lora_wgrad
    gen = torch.Generator().manual_seed(M + 7 * N + R)
    d = torch.randn(M, N, generator=gen).to(torch.bfloat16).cuda()
    r8 = -(-R // 8) * 8  # row stride a multiple of 8 elements: a rank that is not is a column slice
    h = torch.randn(M, r8, generator=gen).to(torch.bfloat16).cuda()[:, :R]
    ref = _reference(d.cpu(), h.cpu(), scale)
    out = lora_wgrad(d, h, scale)
    torch.cuda.synchronize()
    _check(out.cpu(), ref)
    outT = lora_wgrad(d, h, scale, transposed=True)  # [R, N]
    torch.cuda.synchronize()
    assert torch.equal(outT.t().cpu(), out.cpu())


def test_lora_wgrad_strided_operands_and_empty_range():
    """D and H as column slices of wider tensors (row strides past their widths, as the block's
    projection output is sliced), and M = 0 (the gradient of an empty token range is zero)."""
    from recant_b200.block import lora_wgrad
    gen = torch.Generator().manual_seed(5)
    big = torch.randn(2048, 96, generator=gen).to(torch.bfloat16).cuda()
    dwide = torch.randn(2048, 4096 + 64, generator=gen).to(torch.bfloat16).cuda()
    d, h = dwide[:, 64:], big[:, 64:96]
    out = lora_wgrad(d, h, 2.0)
    torch.cuda.synchronize()
    _check(out.cpu(), _reference(d.cpu(), h.cpu(), 2.0))
    empty = lora_wgrad(torch.empty(0, 256, dtype=torch.bfloat16, device="cuda"),
                       torch.empty(0, 16, dtype=torch.bfloat16, device="cuda"), 2.0)
    torch.cuda.synchronize()
    assert empty.shape == (256, 16) and not bool(empty.any())


def test_lora_wgrad_rejects_bad_operands():
    from recant_b200.block import lora_wgrad
    d = torch.randn(128, 256, device="cuda").to(torch.bfloat16)
    with pytest.raises(ValueError):
        lora_wgrad(d, torch.randn(128, 65, device="cuda").to(torch.bfloat16))   # rank above 64
    with pytest.raises(ValueError):
        lora_wgrad(d, torch.randn(128, 16, device="cuda"))                     # fp32 H


def test_block_lora_gradients_kernel_vs_cublas(monkeypatch):
    """The GDN block's output and LoRA gradients (in_proj_qkv, in_proj_z through the grouped addmm
    and the shared down-projection; out_proj through QLinear's three ops) with rb2_lora_up and
    rb2_lora_wgrad against the same forward and backward as the reference's torch ops (cuBLAS), on
    the golden block's input and one upstream gradient (round-to-nearest backward quantization, so
    both runs see the same codes)."""
    import recant_b200.block as blk
    from block_util import HIDDEN, HK, HV, golden

    G = golden()
    sd = {k: v for k, v in G.items() if k not in ("x", "out", "y")}
    block = blk.GDNBlock.from_state(sd, HIDDEN, HK, HV)
    block.set_stochastic_backward(False)
    x = G["x"].to(torch.bfloat16).cuda()
    dy = torch.randn(x.shape, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).cuda()

    def grads(on):
        monkeypatch.setattr(blk, "LORA_WGRAD", on)
        monkeypatch.setattr(blk, "LORA_UP", on)
        for name in ("in_proj_qkv", "in_proj_z", "out_proj"):
            lin = getattr(block, name)
            lin.lora_A.grad = lin.lora_B.grad = None
        xd = x.clone().requires_grad_(True)
        y = block(xd)
        y.backward(dy)
        torch.cuda.synchronize()
        out = {"dx": xd.grad.float().cpu(), "y": y.detach().float().cpu()}
        for name in ("in_proj_qkv", "in_proj_z", "out_proj"):
            lin = getattr(block, name)
            out[name + ".A"] = lin.lora_A.grad.cpu().clone()
            out[name + ".B"] = lin.lora_B.grad.cpu().clone()
        return out

    on, off = grads(True), grads(False)
    assert rel(on["y"], off["y"]) < 1e-2, rel(on["y"], off["y"])
    assert rel(on["dx"], off["dx"]) < 1e-2
    for k in off:
        if k not in ("dx", "y"):
            assert off[k].abs().sum() > 0, k
            assert rel(on[k], off[k]) < 1e-3, (k, rel(on[k], off[k]))


def _up_reference(y, h, b, s, mode):
    acc = (h.double() @ b.double().t()).float()
    if mode == 0:  # torch.addmm on the GPU: the scaled product rounded to bf16, then added
        return (y.float() + (acc * s).to(torch.bfloat16).float()).to(torch.bfloat16)
    t = acc.to(torch.bfloat16)
    return (y.float() + (t.float() * s).to(torch.bfloat16).float()).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,r,mode", [(16384, 4096, 16, 1), (16384, 8192, 16, 0), (1000, 200, 32, 1),
                                        (77, 136, 8, 0), (129, 4096, 64, 1), (300, 256, 48, 0),
                                        (4096, 4096, 96, 1), (300, 256, 128, 0)])
def test_lora_up_matches_reference_ops(M, N, r, mode):
    """rb2_lora_up against the reference's ops on the same bf16 operands: mode 1 (QLinear's three
    ops) and mode 0 (grouped_linear's addmm, which cuBLAS computes as bf16(y + bf16(s acc))) equal a
    float64-accumulated restatement of those roundings within 1e-3 (relative Frobenius), and torch's
    own ops on this GPU element for element (all but 1e-4 of the elements, for fp32 sums that round
    differently)."""
    from recant_b200.block import lora_up
    gen = torch.Generator().manual_seed(M + N + r + mode)
    y = torch.randn(M, N, generator=gen).to(torch.bfloat16).cuda()
    h = torch.randn(M, r, generator=gen).to(torch.bfloat16).cuda()
    b = (torch.randn(N, r, generator=gen) * 0.1).to(torch.bfloat16).cuda()
    out = lora_up(y, h, b, 2.0, mode)
    torch.cuda.synchronize()
    ref = _up_reference(y.cpu(), h.cpu(), b.cpu(), 2.0, mode)
    assert rel(out.float().cpu(), ref.float()) < 1e-3
    torch_ops = torch.addmm(y, h, b.t(), alpha=2.0) if mode == 0 else y + (h @ b.t()) * 2.0
    assert rel(out.float(), torch_ops.float()) < 1e-3
    assert (out == torch_ops).float().mean().item() > 0.9999
    # a strided y (a column slice) and an output row stride equal to N
    if N >= 136:
        wide = torch.randn(M, N + 8, generator=gen).to(torch.bfloat16).cuda()
        y2 = wide[:, 8:]
        out2 = lora_up(y2, h, b, 2.0, mode)
        torch.cuda.synchronize()
        assert rel(out2.float().cpu(), _up_reference(y2.cpu(), h.cpu(), b.cpu(), 2.0, mode).float()) < 1e-3
