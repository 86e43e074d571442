"""The decode step on the GPU: the token-by-token GDN kernel (rb2_gdn_recurrent_fwd) against the CPU
oracle of gdn_torch (ops.py:21-54, one padded chunk) and against the chunked op.

Tolerances (relative Frobenius) as for the chunked op: 1e-4 for fp32 inputs, 2e-2 for bf16 inputs
against the fp32 reference.
"""
import pytest
import torch

from gpu_util import rel
from oracle import gdn as OG
from oracle import inputs as I

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 2e-2


def _state(n, H, seed, scale=0.1):
    return torch.randn(n, H, 128, 128, generator=torch.Generator().manual_seed(seed)) * scale


def _recurrent(inp, h0=None, cu=None):
    from recant_b200 import gdn_recurrent
    d = {n: t.cuda() for n, t in inp.items()}
    o, hT = gdn_recurrent(d["q"], d["k"], d["v"], d["g"], d["beta"], None if h0 is None else h0.cuda(), True,
                          cu_seqlens=None if cu is None else cu.cuda())
    torch.cuda.synchronize()
    return o.cpu(), hT.cpu()


@pytest.mark.parametrize("T", [1, 2, 5, 16, 40])
def test_recurrent_fp32_matches_oracle(T):
    inp = I.gdn_inputs(2, T, 2, 4, 128, dtype=torch.float32, seed=100 + T)
    h0 = _state(2, 4, T)
    ro, rhT = OG.gdn(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], h0, True)
    o, hT = _recurrent(inp, h0)
    assert rel(o, ro) < F32_TOL and rel(hT, rhT) < F32_TOL, (rel(o, ro), rel(hT, rhT))


@pytest.mark.parametrize("Hk,Hv", [(1, 1), (2, 8), (4, 4)])
def test_recurrent_bf16_gqa_matches_oracle(Hk, Hv):
    inp = I.gdn_inputs(3, 7, Hk, Hv, 128, dtype=torch.bfloat16, seed=Hk * 10 + Hv)
    h0 = _state(3, Hv, Hv)
    f32 = {n: t.float() for n, t in inp.items()}
    ro, rhT = OG.gdn(f32["q"], f32["k"], f32["v"], f32["g"], f32["beta"], h0, True)
    o, hT = _recurrent(inp, h0)
    assert o.dtype == torch.bfloat16 and hT.dtype == torch.float32
    assert rel(o.float(), ro) < BF16_TOL and rel(hT, rhT) < BF16_TOL, (rel(o.float(), ro), rel(hT, rhT))


def test_recurrent_without_initial_state():
    inp = I.gdn_inputs(1, 3, 2, 2, 128, dtype=torch.float32, seed=5)
    ro, rhT = OG.gdn(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], None, True)
    o, hT = _recurrent(inp)
    assert rel(o, ro) < F32_TOL and rel(hT, rhT) < F32_TOL


def test_recurrent_varlen_per_sequence_states():
    """cu_seqlens (B = 1): per-sequence initial and final states, as the chunked op's varlen form."""
    lens = [1, 4, 2, 6]
    cu = torch.tensor([0] + torch.cumsum(torch.tensor(lens), 0).tolist(), dtype=torch.int64)
    inp = I.gdn_inputs(1, sum(lens), 2, 4, 128, dtype=torch.float32, seed=9)
    h0 = _state(len(lens), 4, 9)
    ro, rhT = OG.gdn(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], h0, True, cu_seqlens=cu)
    o, hT = _recurrent(inp, h0, cu)
    assert rel(o, ro) < F32_TOL and rel(hT, rhT) < F32_TOL, (rel(o, ro), rel(hT, rhT))


def test_recurrent_agrees_with_chunked_op():
    from recant_b200 import gdn_b200
    inp = {n: t.cuda() for n, t in I.gdn_inputs(2, 16, 2, 4, 128, dtype=torch.float32, seed=21).items()}
    h0 = _state(2, 4, 21).cuda()
    a = gdn_b200(**inp, initial_state=h0, output_final_state=True, path="recurrent")
    b = gdn_b200(**inp, initial_state=h0, output_final_state=True, path="exact")
    assert rel(a[0], b[0]) < F32_TOL and rel(a[1], b[1]) < F32_TOL


def test_auto_dispatch_uses_recurrent_kernel_for_short_no_grad_calls():
    from recant_b200 import _lib as L
    from recant_b200 import gdn_b200
    inp = {n: t.cuda() for n, t in I.gdn_inputs(1, 1, 2, 4, 128, seed=3).items()}
    prof = L.LaunchProfiler(capacity=64)
    prof.start()
    with torch.no_grad():
        gdn_b200(**inp, initial_state=_state(1, 4, 3).cuda(), output_final_state=True)
    torch.cuda.synchronize()
    names = [n for n, _ in prof.read()[0]]
    assert names == ["gdn_recurrent"], names
