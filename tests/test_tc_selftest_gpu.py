"""tcgen05 operand-layout self-test: one-tile products in every K-major / MN-major combination."""
import itertools

import pytest
import torch

from recant_b200 import _lib as L

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("a_mn,b_mn,M,N,K", [c for c in itertools.product((0, 1), (0, 1), (128, 64), (64, 128), (64, 128))])
def test_mma_layouts(a_mn, b_mn, M, N, K):
    gen = torch.Generator().manual_seed(M * 7 + N * 3 + K + 11 * a_mn + 13 * b_mn)
    A = torch.randn(M, K, generator=gen).to(torch.bfloat16)
    B = torch.randn(N, K, generator=gen).to(torch.bfloat16)
    ref = A.float() @ B.float().t()
    Ad = (A.t().contiguous() if a_mn else A).cuda()
    Bd = (B.t().contiguous() if b_mn else B).cuda()
    D = torch.full((M, N), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = L.lib().rb2_selftest_mma(Ad.data_ptr(), Bd.data_ptr(), D.data_ptr(), a_mn, b_mn, M, N, K, err.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    L.check(st, "selftest_mma")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.allclose(D.cpu(), ref, rtol=1e-3, atol=1e-3), (D.cpu() - ref).abs().max()
