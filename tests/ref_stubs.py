"""Stand-ins for the reference's backend registries, used by the registry tests.

They have the shape of the reference modules' dispatch code and nothing else:
* ``<pkg>.model.ops``: ``GDN_BACKENDS``, ``_state['gdn']``, ``set_gdn_backend`` (KeyError on an
  unknown name) and ``gdn_core``, which calls ``GDN_BACKENDS[name](q, k, v, g, beta,
  initial_state=..., output_final_state=...)`` (recant/model/ops.py:5-10,60-67);
* ``<pkg>.model.nvfp4``: ``GEMM_BACKENDS``, ``set_gemm_backend``, ``gemm_fp4`` (nvfp4.py:125-137)
  and the fast-quantizer switch ``_fast`` / ``set_fast_quantizer`` / ``quantize_activation``, which
  imports its sibling ``fp4_kernels`` module lazily and calls ``quantize_fast(x, use_rht,
  stochastic)`` for 2-D CUDA inputs with K % 16 == 0 (nvfp4.py:139-149).
The reference itself is not importable on the GPU box, so GPU tests drive the package's
``register`` functions through these modules; a CPU test also drives the real reference when it
is present.
"""
from __future__ import annotations

import sys
import types

_OPS_SRC = '''
_state = {"gdn": "torch"}

def _unavailable(*a, **k):
    raise RuntimeError("the reference torch op is not part of this stand-in")

GDN_BACKENDS = {"torch": _unavailable}

def set_gdn_backend(name):
    if name not in GDN_BACKENDS:
        raise KeyError(f"unknown GDN backend {name!r}; have {list(GDN_BACKENDS)}")
    _state["gdn"] = name

def get_gdn_backend():
    return _state["gdn"]

def gdn_core(q, k, v, g, beta, initial_state=None, output_final_state=False):
    return GDN_BACKENDS[_state["gdn"]](q, k, v, g, beta, initial_state=initial_state,
                                       output_final_state=output_final_state)
'''

_NVFP4_SRC = '''
BLOCK = 16

def _emulated(a, b):
    raise RuntimeError("the reference emulated GEMM is not part of this stand-in")

GEMM_BACKENDS = {"emulated": _emulated}
_state = {"gemm": "emulated"}

def set_gemm_backend(name):
    if name not in GEMM_BACKENDS:
        raise KeyError(f"unknown FP4 GEMM backend {name!r}; have {list(GEMM_BACKENDS)}")
    _state["gemm"] = name

def gemm_fp4(a, b):
    return GEMM_BACKENDS[_state["gemm"]](a, b)

_fast = {"quantize": False}

def set_fast_quantizer(flag):
    _fast["quantize"] = bool(flag)

def quantize_activation(x, use_rht=True, stochastic=False):
    if _fast["quantize"] and x.is_cuda and x.dim() == 2 and x.shape[1] % BLOCK == 0:
        from . import fp4_kernels
        return fp4_kernels.quantize_fast(x.contiguous(), use_rht, stochastic)
    raise RuntimeError("the reference CPU quantizer is not part of this stand-in")
'''


def make_reference_stubs(pkg: str):
    """Create ``pkg``, ``pkg.model``, ``pkg.model.ops`` and ``pkg.model.nvfp4`` in sys.modules and
    return (ops, nvfp4). Call :func:`drop_reference_stubs` afterwards."""
    top = types.ModuleType(pkg)
    top.__path__ = []
    model = types.ModuleType(pkg + ".model")
    model.__path__ = []
    top.model = model
    sys.modules[pkg] = top
    sys.modules[pkg + ".model"] = model
    mods = []
    for name, src in (("ops", _OPS_SRC), ("nvfp4", _NVFP4_SRC)):
        m = types.ModuleType(f"{pkg}.model.{name}")
        m.__package__ = pkg + ".model"
        exec(compile(src, f"<{pkg}.model.{name}>", "exec"), m.__dict__)
        sys.modules[m.__name__] = m
        setattr(model, name, m)
        mods.append(m)
    return tuple(mods)


def drop_reference_stubs(pkg: str) -> None:
    for name in [n for n in sys.modules if n == pkg or n.startswith(pkg + ".")]:
        del sys.modules[name]
