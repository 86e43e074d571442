"""recant_b200: B200-native (sm_100a) chunked Gated DeltaNet + NVFP4 hot path of RECANT.

The compute lives in the in-tree CUDA library ``recant_b200/_lib/librecant_b200.so``
(C ABI in include/recant_b200.h, built by ``python -m recant_b200.build``); this package is the
host side that mirrors the reference's backend registries (recant/model/ops.py and
recant/model/nvfp4.py) so the reference's callers can use it unchanged.
"""
from . import _lib
from ._lib import DeviceStatusError, set_status_checks
from .gdn import GDN_BACKENDS, gdn_b200, gdn_core, gdn_recurrent, get_gdn_backend, set_gdn_backend
from .nvfp4 import FP4Tensor, gemm_b200, quantize_activation, quantize_fast
from .segmented import gdn_segmented

__all__ = ["GDN_BACKENDS", "gdn_b200", "gdn_core", "gdn_recurrent", "get_gdn_backend", "set_gdn_backend", "FP4Tensor",
           "gemm_b200", "quantize_activation", "quantize_fast", "gdn_segmented", "set_status_checks",
           "DeviceStatusError"]


def library_version() -> str:
    return _lib.lib().rb2_version().decode()
