"""NVFP4 block-scaled GEMM parity: tcgen05 kind::mxf4nvf4 vs the emulated reference GEMM
(dequantise both operands, fp32 matmul; recant/model/nvfp4.py:108-110). Tolerance 5e-3 relative
Frobenius (the reference's own check, recant/backends.py:21-35, allows 3e-2)."""
import random

import numpy as np
import pytest
import torch

from oracle import nvfp4 as ON

pytestmark = pytest.mark.gpu
TOL = 5e-3


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _fp4(x_gpu, rht=True):
    from recant_b200 import quantize_fast
    return quantize_fast(x_gpu, rht, False)


def _oracle(t, k):
    return (t.codes.cpu().numpy(), t.scales.view(torch.uint8).cpu().numpy(), float(t.gscale.cpu()), (t.shape[0], k))


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (300, 2048, 1024), (257, 384, 320), (64, 100, 64), (512, 1024, 4096)])
def test_gemm_matches_emulated(M, N, K):
    from recant_b200 import gemm_b200
    gen = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=gen) * 0.05).to(torch.bfloat16).cuda()
    a, b = _fp4(x), _fp4(w)
    out = gemm_b200(a, b).cpu().numpy()
    ref = ON.gemm_emulated(_oracle(a, K), _oracle(b, K))
    assert _rel(out, ref) < TOL, _rel(out, ref)
    out16 = gemm_b200(a, b, out_dtype=torch.bfloat16).float().cpu().numpy()
    assert _rel(out16, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (300, 2048, 1024), (257, 384, 320), (64, 100, 64), (512, 1024, 4096)])
def test_gemm_pair_matches_emulated_and_one_sm(M, N, K):
    """The SM-pair kernel (cta_group::2, 256 x 256 tiles): rows past M, columns past N and a ragged
    last K stage as above; against the emulated GEMM and against the one-SM kernel's output."""
    from recant_b200 import gemm_b200
    from recant_b200.nvfp4 import gemm_pair_b200
    gen = torch.Generator().manual_seed(M + N + K + 1)
    x = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=gen) * 0.05).to(torch.bfloat16).cuda()
    a, b = _fp4(x), _fp4(w)
    out = gemm_pair_b200(a, b)
    ref = ON.gemm_emulated(_oracle(a, K), _oracle(b, K))
    assert _rel(out.cpu().numpy(), ref) < TOL
    one = gemm_b200(a, b)
    assert _rel(out.cpu().numpy(), one.cpu().numpy()) < 1e-6
    out16 = gemm_pair_b200(a, b, out_dtype=torch.bfloat16).float().cpu().numpy()
    assert _rel(out16, ref) < 1e-2


def test_gemm_on_reference_layout_scales():
    """Operands without pre-blocked scales (e.g. quantized by the reference) get blocked on the GPU."""
    from recant_b200 import nvfp4 as N
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(200, 512, generator=gen)
    c, s, g = ON.quantize_activation(x.numpy(), "f32", True)
    t = N.FP4Tensor(torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda().view(torch.float8_e4m3fn),
                    torch.tensor(g).cuda(), (200, 512))
    out = N.gemm_b200(t, t).cpu().numpy()
    ref = ON.gemm_emulated((c, s, g, (200, 512)), (c, s, g, (200, 512)))
    assert _rel(out, ref) < TOL


def test_reference_select_fp4_gemm_check():
    """The reference's backend check (recant/backends.py:21-35): fprop and dgrad at 300x1024 @ 2048x1024
    against the emulated GEMM, rel err < 0.03."""
    from recant_b200 import nvfp4 as N
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(300, 1024, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(2048, 1024, generator=gen) * 0.05).to(torch.bfloat16).cuda()
    W = N.quantize_weight(w)
    a = N.quantize_fast(x, True, False)
    e1 = _rel(N.gemm_b200(a, W.fprop).cpu().numpy(), ON.gemm_emulated(_oracle(a, 1024), _oracle(W.fprop, 1024)))
    dy = torch.randn(300, 2048, generator=gen).to(torch.bfloat16).cuda()
    d = N.quantize_fast(dy, True, True)
    e2 = _rel(N.gemm_b200(d, W.dgrad).cpu().numpy(), ON.gemm_emulated(_oracle(d, 2048), _oracle(W.dgrad, 2048)))
    assert e1 < 0.03 and e2 < 0.03 and e1 < TOL and e2 < TOL, (e1, e2)


def test_quantize_weight_bit_exact():
    """GPU quantize_weight equals the reference's (fp32 RHT, fprop and dgrad copies)."""
    from recant_b200 import nvfp4 as N
    gen = torch.Generator().manual_seed(21)
    w = torch.randn(512, 256, generator=gen) * 0.02
    W = N.quantize_weight(w.cuda())
    fp, dg = ON.quantize_weight(w.numpy())
    assert np.array_equal(W.fprop.codes.cpu().numpy(), fp[0]) and np.array_equal(W.dgrad.codes.cpu().numpy(), dg[0])
    assert np.array_equal(W.fprop.scales.view(torch.uint8).cpu().numpy(), fp[1])
    assert float(W.dgrad.gscale.cpu()) == float(dg[2])


def test_fp4_linear_fwd_bwd():
    """FP4Linear: forward = RN-quantized activations through fprop; backward = SR-quantized dy through dgrad."""
    from recant_b200 import nvfp4 as N
    gen = torch.Generator().manual_seed(5)
    w = (torch.randn(512, 256, generator=gen) * 0.02).cuda()
    W = N.quantize_weight(w)
    x = torch.randn(4, 32, 256, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    y = N.fp4_linear(x, W)
    ref = ON.gemm_emulated(_oracle(N.quantize_fast(x.detach().reshape(-1, 256), True, False), 256), _oracle(W.fprop, 256))
    assert _rel(y.detach().float().reshape(-1, 512).cpu().numpy(), ref) < 1e-2
    dy = torch.randn(4, 32, 512, generator=gen).to(torch.bfloat16).cuda()
    random.seed(1234)  # the backward's stochastic-rounding seed comes from random.getrandbits
    y.backward(dy)
    exact = (dy.float().reshape(-1, 512) @ w.float()).cpu().numpy()
    # against the exact product: within NVFP4's own quantization error
    assert x.grad.shape == x.shape and _rel(x.grad.float().reshape(-1, 256).cpu().numpy(), exact) < 0.2
    # against the same SR codes (re-drawn with the same seed) through the emulated GEMM: the dgrad
    # itself, pinned at the bf16 output rounding
    random.seed(1234)
    d = N.quantize_fast(dy.reshape(-1, 512), True, True)
    ref_dx = ON.gemm_emulated(_oracle(d, 512), _oracle(W.dgrad, 512))
    assert _rel(x.grad.float().reshape(-1, 256).cpu().numpy(), ref_dx) < 5e-3
    assert torch.equal(x.grad.reshape(-1, 256), N.gemm_b200(d, W.dgrad, out_dtype=torch.bfloat16))


@pytest.mark.parametrize("M,N,K", [(257, 384, 320), (1, 4096, 4096), (64, 100, 64)])
def test_gemm_with_cached_weight_images_is_identical(M, N, K):
    """B's scales kept on the weight (gemm_images), or copied once through rb2_nvfp4_gemm_b_images and
    passed as the precomputed B operand, give bit-for-bit the result of the plain call."""
    from recant_b200 import _lib as L
    from recant_b200 import gemm_b200
    from recant_b200.nvfp4 import blocked_scales, gemm_images
    gen = torch.Generator().manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=gen) * 0.05).to(torch.bfloat16).cuda()
    a, b = _fp4(x), _fp4(w)
    plain = gemm_b200(a, b)
    gemm_images(b)
    assert b.gemm_images is not None
    cached = gemm_b200(a, b)
    assert torch.equal(plain, cached)
    lib = L.lib()
    nb = lib.rb2_nvfp4_gemm_b_images_size(N, K)
    img = torch.full((nb,), 0xAB, dtype=torch.uint8, device="cuda")
    L.check(lib.rb2_nvfp4_gemm_b_images(L.ptr(blocked_scales(b)), N, K, L.ptr(img), nb,
                                        torch.cuda.current_stream().cuda_stream), "nvfp4_gemm_b_images")
    b.gemm_images = img
    copied = gemm_b200(a, b)
    assert torch.equal(plain, copied)


@pytest.mark.parametrize("M,N,K,r", [(300, 512, 256, 16), (257, 384, 320, 8), (1, 4096, 1024, 16)])
def test_gemm_lora_epilogue(M, N, K, r):
    """out = a . b^T gA gB + s h B^T with the low-rank term added in the GEMM epilogue, against the
    plain GEMM plus the same term in fp32."""
    from recant_b200 import gemm_b200
    gen = torch.Generator().manual_seed(M + 3 * N + r)
    x = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=gen) * 0.05).to(torch.bfloat16).cuda()
    hfull = torch.randn(M, 2 * r, generator=gen).to(torch.bfloat16).cuda()
    h = hfull[:, r:]                       # a column slice: row stride 2r
    Bm = (torch.randn(N, r, generator=gen) * 0.3).to(torch.bfloat16).cuda()
    a, b = _fp4(x), _fp4(w)
    base = gemm_b200(a, b)
    ref = base + 2.0 * (h.float() @ Bm.float().t())
    out = gemm_b200(a, b, lora=(h, Bm, 2.0))
    assert _rel(out.cpu().numpy(), ref.cpu().numpy()) < 1e-6
    out16 = gemm_b200(a, b, out_dtype=torch.bfloat16, lora=(h, Bm, 2.0))
    assert _rel(out16.float().cpu().numpy(), ref.cpu().numpy()) < 5e-3
    # bf16 output against grouped_linear's own op on this GPU, torch.addmm over the bf16 base output
    # (the low-rank sum runs on CUDA cores here, in another order: a few elements may round apart)
    addmm = torch.addmm(base.to(torch.bfloat16), h, Bm.t(), alpha=2.0)
    assert (out16 == addmm).float().mean().item() > 0.995


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (2, 300, 512), (3, 12288, 1024), (4, 7, 32), (1, 129, 4128)])
def test_gemv_matches_emulated_and_tensor_core_gemm(M, N, K):
    """rb2_nvfp4_gemv (M <= 4, the decode step) against the emulated reference GEMM and against the
    tensor-core kernel on the same operands (that path forced with GEMV_MAX_M = 0)."""
    from recant_b200 import _lib as L
    from recant_b200 import gemm_b200
    from recant_b200 import nvfp4 as N_
    gen = torch.Generator().manual_seed(M * 1000 + N + K)
    x = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=gen) * 0.05).to(torch.bfloat16).cuda()
    a, b = _fp4(x), _fp4(w)
    prof = L.LaunchProfiler(capacity=64)
    prof.start()
    out = gemm_b200(a, b)
    out16 = gemm_b200(a, b, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert {n for n, _ in prof.read()[0]} == {"nvfp4_gemv"}
    ref = ON.gemm_emulated(_oracle(a, K), _oracle(b, K))
    assert _rel(out.cpu().numpy(), ref) < 1e-5, _rel(out.cpu().numpy(), ref)
    assert _rel(out16.float().cpu().numpy(), ref) < 1e-2
    if K % 64 == 0:
        old = N_.GEMV_MAX_M
        try:
            N_.GEMV_MAX_M = 0
            tc_out = gemm_b200(a, b)
        finally:
            N_.GEMV_MAX_M = old
        assert _rel(out.cpu().numpy(), tc_out.cpu().numpy()) < 1e-5


def test_gemm_config2_in_proj_shape():
    """The fused in_proj fprop of the block benchmark at full size: A = Q(rht(x)) for x [16384, 4096]
    bf16 ~ N(0, 1), B = the fprop copy of a [12288, 4096] weight ~ N(0, 0.02) from quantize_weight
    (qkv 8192 rows + z 4096 rows). The whole 16384 x 12288 product runs on the GPU (every output tile
    of the persistent schedule); 256 rows drawn from the first, middle and last row tiles are checked
    against the emulated GEMM of those rows."""
    from recant_b200 import gemm_b200, quantize_fast
    from recant_b200 import nvfp4 as N
    M, Nn, K = 16384, 12288, 4096
    gen = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(M, K, device="cuda", generator=gen).to(torch.bfloat16)
    W = N.quantize_weight(torch.randn(Nn, K, device="cuda", generator=gen) * 0.02)
    a = quantize_fast(x, True, False)
    out = gemm_b200(a, W.fprop)
    rows = torch.cat([torch.arange(0, 64), torch.arange(M // 2 - 64, M // 2 + 64), torch.arange(M - 64, M)])
    ac = a.codes[rows.cuda()].cpu().numpy()
    asc = a.scales.view(torch.uint8)[rows.cuda()].cpu().numpy()
    ref = ON.gemm_emulated((ac, asc, float(a.gscale.cpu()), (len(rows), K)), _oracle(W.fprop, K))
    got = out[rows.cuda()].cpu().numpy()
    assert _rel(got, ref) < TOL, _rel(got, ref)
    out16 = gemm_b200(a, W.fprop, out_dtype=torch.bfloat16)[rows.cuda()].float().cpu().numpy()
    assert _rel(out16, ref) < 1e-2
