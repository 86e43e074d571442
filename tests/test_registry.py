"""The package's register() functions plug into the reference's backend registries (CPU).

``recant_b200.gdn.register`` adds 'b200' to ``ops.GDN_BACKENDS`` (recant/model/ops.py:60-67) and
``recant_b200.nvfp4.register`` adds it to ``nvfp4.GEMM_BACKENDS`` (nvfp4.py:125-137) and installs
the fast quantizer hook behind ``nvfp4._fast`` (nvfp4.py:139-149). On the CPU the ops themselves
refuse CPU tensors, so a call routed through the registry that ends in this package's error shows
that the dispatch reached it. Driven through stand-ins shaped like the reference's modules and,
when the reference checkout is present, through the reference itself.
"""
import os
import sys

import pytest
import torch

from ref_stubs import drop_reference_stubs, make_reference_stubs

REF = "/root/reference"


def _gdn_args():
    q = torch.randn(1, 64, 2, 128)
    v = torch.randn(1, 64, 2, 128)
    return q, q.clone(), v, -torch.rand(1, 64, 2), torch.rand(1, 64, 2)


def _check_gdn_registry(ops):
    from recant_b200 import gdn as G
    G.register(ops)
    assert ops.GDN_BACKENDS["b200"] is G.gdn_b200
    assert ops.get_gdn_backend() != "b200"           # registering does not select
    G.register(ops, select=True)
    assert ops.get_gdn_backend() == "b200"
    with pytest.raises(ValueError, match="recant_b200.gdn: inputs must be CUDA tensors"):
        ops.gdn_core(*_gdn_args(), initial_state=None, output_final_state=True)


def _check_nvfp4_registry(nv):
    from recant_b200 import nvfp4 as N
    N.register(nv, select=True)
    assert nv.GEMM_BACKENDS["b200"] is N.gemm_b200
    assert nv._state["gemm"] == "b200"
    assert nv._fast["quantize"] is True
    kernels = sys.modules[nv.__name__.rpartition(".")[0] + ".fp4_kernels"]
    assert kernels.quantize_fast is N.quantize_fast
    a = N.FP4Tensor(torch.zeros(4, 8, dtype=torch.uint8), torch.zeros(4, 1, dtype=torch.uint8),
                    torch.ones(()), (4, 16))
    with pytest.raises(ValueError, match="recant_b200.gemm_b200: operands must be CUDA tensors"):
        nv.gemm_fp4(a, a)
    with pytest.raises(ValueError, match="recant_b200.quantize_fast"):
        kernels.quantize_fast(torch.zeros(4, 16), True, False)


def test_register_into_reference_shaped_registries():
    ops, nv = make_reference_stubs("refstub_cpu")
    try:
        _check_gdn_registry(ops)
        _check_nvfp4_registry(nv)
        with pytest.raises(KeyError):
            ops.set_gdn_backend("no-such-backend")
    finally:
        drop_reference_stubs("refstub_cpu")


def test_recurrent_path_refuses_inputs_that_need_grad():
    """The forward-only recurrent kernel is never taken silently for a training call."""
    from recant_b200 import gdn_b200
    q, k, v, g, beta = _gdn_args()
    q.requires_grad_(True)
    with pytest.raises(ValueError, match="forward-only"):
        gdn_b200(q, k, v, g, beta, path="recurrent")


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "recant")), reason="reference checkout not present")
def test_register_into_the_reference_itself():
    saved_path = list(sys.path)
    before = set(sys.modules)
    sys.path.insert(0, REF)
    try:
        from recant.model import nvfp4 as ref_nvfp4
        from recant.model import ops as ref_ops
        _check_gdn_registry(ref_ops)
        _check_nvfp4_registry(ref_nvfp4)
        # the reference's own default backend is still selectable afterwards
        ref_ops.set_gdn_backend("torch")
        ref_nvfp4.set_gemm_backend("emulated")
        ref_nvfp4.set_fast_quantizer(False)
    finally:
        sys.path[:] = saved_path
        for name in set(sys.modules) - before:
            if name == "recant" or name.startswith("recant."):
                del sys.modules[name]
