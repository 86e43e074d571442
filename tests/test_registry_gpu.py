"""Calls through the reference's registries reach this package's kernels and give what a direct
call gives (GPU). The reference does not travel to the GPU box, so its dispatch is driven through
stand-ins shaped like recant/model/ops.py:60-67 and recant/model/nvfp4.py:125-149
(tests/ref_stubs.py): ``ops.gdn_core`` -> ``GDN_BACKENDS['b200']``, ``nvfp4.gemm_fp4`` ->
``GEMM_BACKENDS['b200']`` and ``nvfp4.quantize_activation`` -> the installed fast quantizer hook."""
import pytest
import torch

from oracle import gdn as OG
from oracle import inputs as I
from gpu_util import rel
from ref_stubs import drop_reference_stubs, make_reference_stubs

pytestmark = pytest.mark.gpu


@pytest.fixture
def ref():
    ops, nv = make_reference_stubs("refstub_gpu")
    yield ops, nv
    drop_reference_stubs("refstub_gpu")


def test_gdn_through_reference_registry(ref):
    from recant_b200 import gdn as G
    ops, _ = ref
    G.register(ops, select=True)
    inp = I.gdn_inputs(1, 200, 2, 2, 128, dtype=torch.bfloat16, seed=31)
    d = {n: t.cuda() for n, t in inp.items()}
    with torch.no_grad():
        o_reg, h_reg = ops.gdn_core(d["q"], d["k"], d["v"], d["g"], d["beta"], initial_state=None,
                                    output_final_state=True)
        o_dir, h_dir = G.gdn_b200(d["q"], d["k"], d["v"], d["g"], d["beta"], None, True)
    torch.cuda.synchronize()
    assert torch.equal(o_reg, o_dir) and torch.equal(h_reg, h_dir)
    f32 = {n: t.float() for n, t in inp.items()}
    ro, rh = OG.gdn(f32["q"], f32["k"], f32["v"], f32["g"], f32["beta"], None, True)
    assert rel(o_reg, ro) < 2e-2 and rel(h_reg, rh) < 2e-2


def test_nvfp4_through_reference_registry(ref):
    from recant_b200 import nvfp4 as N
    _, nv = ref
    N.register(nv, select=True)
    gen = torch.Generator().manual_seed(5)
    x = (torch.randn(256, 512, generator=gen) * 2).to(torch.bfloat16).cuda()
    w = (torch.randn(384, 512, generator=gen) * 0.05).to(torch.bfloat16).cuda()
    a_reg = nv.quantize_activation(x, True, False)          # through the installed hook
    a_dir = N.quantize_fast(x, True, False)
    b = N.quantize_fast(w, True, False)
    for f in ("codes", "scales", "gscale"):
        assert torch.equal(getattr(a_reg, f).view(torch.uint8) if f == "scales" else getattr(a_reg, f),
                           getattr(a_dir, f).view(torch.uint8) if f == "scales" else getattr(a_dir, f))
    y_reg = nv.gemm_fp4(a_reg, b)
    y_dir = N.gemm_b200(a_dir, b)
    torch.cuda.synchronize()
    assert y_reg.dtype == torch.float32 and torch.equal(y_reg, y_dir)
