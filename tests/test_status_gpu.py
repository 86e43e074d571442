"""Device status words: the bounded waits of the library's kernels give up, record a code and return
(the reference's wrapper contract: device-side guards write an error word that the wrapper checks).
The self-test makes one wait run out on purpose (an mbarrier that nothing completes), then the
context must work as before; with status checks on, the wrappers read each op's word and raise."""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _gdn_case():
    from recant_b200 import gdn_b200
    gen = torch.Generator().manual_seed(21)
    B, T, Hk, Hv, d = 1, 200, 2, 4, 128
    q = torch.randn(B, T, Hk, d, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    k = torch.randn(B, T, Hk, d, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    v = torch.randn(B, T, Hv, d, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    g = (-torch.rand(B, T, Hv, generator=gen) * 0.1).cuda().requires_grad_(True)
    beta = torch.rand(B, T, Hv, generator=gen).to(torch.bfloat16).cuda().requires_grad_(True)
    o, _ = gdn_b200(q, k, v, g, beta)
    o.backward(torch.ones_like(o))
    torch.cuda.synchronize()
    return [o.detach().clone()] + [t.grad.clone() for t in (q, k, v, g, beta)]


def test_bounded_wait_runs_out_records_its_code_and_the_context_survives():
    from recant_b200 import _lib as L
    before = _gdn_case()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    L.check(L.lib().rb2_selftest_wait(status.data_ptr(), 1 << 14, stream), "selftest_wait")
    torch.cuda.synchronize()
    assert int(status.item()) == 901  # the completed barrier passed (no 902), the other one gave up
    code = C.c_int(-1)
    L.check(L.lib().rb2_status_read(status.data_ptr(), C.byref(code), 1, stream), "status_read")
    assert code.value == 901 and int(status.item()) == 0  # read, then cleared
    after = _gdn_case()  # the same op after the timed-out kernel: bit-identical results
    assert all(torch.equal(a, b) for a, b in zip(before, after))


def test_status_checks_pass_on_real_calls():
    import recant_b200
    from recant_b200 import gemm_b200, quantize_fast
    from recant_b200.block import narrow_product
    recant_b200.set_status_checks(True)
    try:
        _gdn_case()
        x = torch.randn(300, 512, device="cuda").to(torch.bfloat16)
        w = (torch.randn(256, 512, device="cuda") * 0.05).to(torch.bfloat16)
        gemm_b200(quantize_fast(x, True, False), quantize_fast(w, True, False))
        xs = torch.randn(4096, 512, device="cuda").to(torch.bfloat16)
        narrow_product(xs, torch.randn(64, 512, device="cuda").to(torch.bfloat16))
    finally:
        recant_b200.set_status_checks(False)


def test_status_check_raises_on_a_recorded_code():
    import recant_b200
    from recant_b200 import _lib as L
    word = torch.zeros(64, dtype=torch.uint8, device="cuda")
    word[:4].view(torch.int32).fill_(901)
    L.check_status(word, "test")  # checks off: nothing is read
    recant_b200.set_status_checks(True)
    try:
        with pytest.raises(recant_b200.DeviceStatusError) as e:
            L.check_status(word, "test")
        assert e.value.code == 901
    finally:
        recant_b200.set_status_checks(False)
