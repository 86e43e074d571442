"""rb2_skinny_gemm (the block's narrow projections of x on tcgen05) against a float64 matmul of the
same bf16 operands: fp32 output within 1e-5 relative Frobenius, bf16 output within 8e-3."""
import pytest
import torch

from gpu_util import rel

pytestmark = pytest.mark.gpu


def _run(a, w, out_dtype, lda=None):
    from recant_b200 import _lib as L
    M, K = a.shape[0], w.shape[1]
    N = w.shape[0]
    out = torch.empty(M, N, dtype=out_dtype, device="cuda")
    st = L.lib().rb2_skinny_gemm(a.data_ptr(), lda or a.stride(0), w.data_ptr(), M, N, K, out.data_ptr(), N,
                                 L.BF16 if out_dtype == torch.bfloat16 else L.F32,
                                 torch.cuda.current_stream().cuda_stream)
    L.check(st, "skinny_gemm")
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("M,N,K", [(300, 96, 4096), (128, 16, 64), (1, 48, 256), (777, 256, 512), (64, 32, 192)])
def test_skinny_gemm_matches_matmul(M, N, K):
    gen = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=gen).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=gen) * 0.05).to(torch.bfloat16).cuda()
    ref = a.double() @ w.double().t()
    assert rel(_run(a, w, torch.float32), ref) < 1e-5
    assert rel(_run(a, w, torch.bfloat16), ref) < 8e-3


def test_skinny_gemm_strided_rows_and_full_block_shape():
    """A as a column slice of a wider tensor (row stride > K), and the block shape: 16384 rows of a
    4096-wide activation against the 96 concatenated b / a / LoRA-A rows."""
    gen = torch.Generator().manual_seed(9)
    big = torch.randn(16384, 4096 + 64, generator=gen).to(torch.bfloat16).cuda()
    a = big[:, 64:]
    w = (torch.randn(96, 4096, generator=gen) * 0.02).to(torch.bfloat16).cuda()
    out = _run(a, w, torch.float32, lda=big.stride(0))
    rows = torch.cat([torch.arange(0, 128), torch.arange(8000, 8128), torch.arange(16384 - 128, 16384)]).cuda()
    ref = a[rows].double() @ w.double().t()
    assert rel(out[rows], ref) < 1e-5


def test_skinny_gemm_rejects_bad_shapes():
    from recant_b200 import _lib as L
    a = torch.zeros(64, 128, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(24, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(64, 24, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert L.lib().rb2_skinny_gemm(a.data_ptr(), 128, w.data_ptr(), 64, 24, 128, out.data_ptr(), 24, L.F32, s) == L.EINVAL
    assert L.lib().rb2_skinny_gemm(a.data_ptr(), 128, w.data_ptr(), 64, 16, 100, out.data_ptr(), 24, L.F32, s) == L.EINVAL
