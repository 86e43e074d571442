"""ctypes binding of the in-tree CUDA library (``recant_b200/_lib/librecant_b200.so``).

The library has a plain C ABI (include/recant_b200.h); this module declares every entry point's
argument types and turns non-zero status codes into Python exceptions. There is no fallback:
if the library is missing, every op raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "librecant_b200.so")

OK, EINVAL, EUNSUPPORTED, ECUDA, EWORKSPACE, ENOMEM, EDEVICE = range(7)
F32, BF16 = 0, 1
GDN_AUTO, GDN_EXACT, GDN_FAST = 0, 1, 2

_p, _i, _i64, _u64, _sz, _f = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_size_t, C.c_float

SIGNATURES = {
    "rb2_last_error": (C.c_char_p, []),
    "rb2_version": (C.c_char_p, []),
    "rb2_gdn_workspace_size": (_sz, [_i64, _i64, _i64, _i, _i, _i, _i, _i, _i]),
    "rb2_gdn_workspace_split": (_i, [_i64, _i64, _i64, _i, _i, _i, _i, _i, _i, C.POINTER(_sz), C.POINTER(_sz)]),
    "rb2_gdn_fwd": (_i, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _i, _i, _f,
                         _p, _p, _p, _sz, _p]),
    "rb2_gdn_bwd": (_i, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _i, _i, _f,
                         _p, _p, _p, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "rb2_gdn_fwd_ex": (_i, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _i, _i, _f,
                            _p, _p, _p, _sz, _p, _i, _i]),
    "rb2_gdn_bwd_ex": (_i, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _i, _i, _f,
                            _p, _p, _p, _p, _p, _p, _p, _p, _p, _sz, _p, _sz, _p, _i, _i]),
    "rb2_gdn_state_fold": (_i, [_p, _p, _p, _i64, _i, _i, _i, _i, _p, _p, _p]),
    "rb2_gdn_state_fold_ex": (_i, [_p, _p, _i64, _p, _p, _i64, _p, _i, _i, _i, _i, _p, _p, _p]),
    "rb2_gdn_recurrent_fwd": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _i, _f, _p, _p, _p]),
    "rb2_conv_silu_fwd": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p, _p, _i, _i, _p, _p]),
    "rb2_conv_silu_bwd": (_i, [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _p]),
    "rb2_gdn_gates_fwd": (_i, [_p, _p, _p, _p, _i64, _i, _p, _p, _p]),
    "rb2_gdn_gates_bwd": (_i, [_p, _p, _p, _p, _p, _p, _i64, _i, _p, _p, _p]),
    "rb2_gated_rmsnorm_fwd": (_i, [_p, _p, _p, _i64, _i, _f, _p, _p, _p]),
    "rb2_gated_rmsnorm_bwd": (_i, [_p, _p, _p, _p, _p, _i64, _i, _p, _p, _p]),
    "rb2_nvfp4_quantize_workspace_size": (_sz, [_i64, _i64]),
    "rb2_nvfp4_quantize": (_i, [_p, _i64, _i64, _i, _i, _i, _u64, _p, _p, _p, _p, _p, _sz, _p]),
    "rb2_nvfp4_quantize_noalloc": (_i, [_p, _i64, _i64, _i, _i, _i, _u64, _p, _p, _p, _p, _p]),
    "rb2_nvfp4_block_scales": (_i, [_p, _i64, _i64, _p, _p]),
    "rb2_nvfp4_gemm_workspace_size": (_sz, [_i64, _i64, _i64]),
    "rb2_nvfp4_gemm": (_i, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _i, _p, _sz, _p]),
    "rb2_nvfp4_gemm_pair": (_i, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _i, _p, _sz, _p]),
    "rb2_status_read": (_i, [_p, C.POINTER(_i), _i, _p]),
    "rb2_skinny_gemm_status": (_i, [C.POINTER(_i), _i]),
    "rb2_selftest_wait": (_i, [_p, C.c_uint, _p]),
    "rb2_nvfp4_gemm_ex": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _i, _f, _i, _i64, _i64, _i64, _p, _i, _p,
                               _sz, _p]),
    "rb2_nvfp4_gemm_b_images_size": (_sz, [_i64, _i64]),
    "rb2_nvfp4_gemv": (_i, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _i, _p]),
    "rb2_nvfp4_gemm_b_images": (_i, [_p, _i64, _i64, _p, _sz, _p]),
    "rb2_skinny_gemm": (_i, [_p, _i64, _p, _i64, _i64, _i64, _p, _i64, _i, _p]),
    "rb2_lora_up_workspace_size": (_sz, []),
    "rb2_lora_up": (_i, [_p, _i64, _p, _i64, _p, _i64, _i64, _i64, _i, _f, _i, _p, _i64, _p, _sz, _p]),
    "rb2_lora_wgrad_workspace_size": (_sz, [_i64, _i64, _i]),
    "rb2_lora_wgrad": (_i, [_p, _i64, _p, _i64, _i64, _i64, _i, _f, _p, _i64, _i64, _p, _sz, _p]),
    "rb2_gated_rmsnorm_nvfp4_fwd": (_i, [_p, _p, _p, _i64, _i, _f, _p, _p, _i64, _i64, _i, _p, _p, _p, _p, _p, _sz,
                                         _p]),
    "rb2_profile_enable": (_i, [_i]),
    "rb2_profile_disable": (_i, []),
    "rb2_profile_read": (_i, [_i, C.c_char_p, _sz, C.POINTER(C.c_float)]),
    "rb2_profile_dropped": (_i, []),
    "rb2_selftest_mma": (_i, [_p, _p, _p, _i, _i, _i, _i, _i, _p, _p]),
}

_lock = threading.Lock()
_lib = None


class LibraryError(RuntimeError):
    """A recant_b200 entry point returned a non-zero status."""


def lib() -> C.CDLL:
    """Load the library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"recant_b200 CUDA library not built: {LIB_PATH} is missing "
                                      "(run `python -m recant_b200.build`)")
                h = C.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.restype, fn.argtypes = res, args
                _lib = h
    return _lib


def check(status: int, what: str) -> None:
    if status == OK:
        return
    msg = lib().rb2_last_error().decode(errors="replace")
    if status == ENOMEM or "out of memory" in msg:
        import torch
        raise torch.cuda.OutOfMemoryError(f"recant_b200 {what}: {msg}")
    raise LibraryError(f"recant_b200 {what} failed (status {status}): {msg}")


# Device status words. Every bounded wait in the library's kernels gives up after a limit instead of
# spinning for ever, records a code in its op's status word (the first 4 bytes of the op's workspace;
# the narrow projection's is a device variable) and lets the kernel finish. Reading a word
# synchronises, so the wrappers read them only when status checks are on.
_status_checks = [False]


def set_status_checks(on: bool) -> None:
    """After every GDN, NVFP4 GEMM and narrow-projection call, read the op's device status word
    (synchronising the stream) and raise DeviceStatusError if a bounded wait ran out."""
    _status_checks[0] = bool(on)


def status_checks() -> bool:
    return _status_checks[0]


class DeviceStatusError(RuntimeError):
    """A bounded device wait ran out: the kernel recorded ``code`` and returned without finishing."""

    def __init__(self, what: str, code: int):
        super().__init__(f"recant_b200 {what}: a bounded device wait ran out (code {code}); the kernel "
                         f"returned early and its outputs are not valid")
        self.code = code


def check_status(ws, what: str) -> None:
    """Raise DeviceStatusError if the status word at the start of ``ws`` (a device tensor holding an
    op's workspace) is non-zero. Only when status checks are on."""
    if not _status_checks[0]:
        return
    code = C.c_int(0)
    check(lib().rb2_status_read(ws.data_ptr(), C.byref(code), 0, _current_stream(ws)), "status_read")
    if code.value:
        raise DeviceStatusError(what, code.value)


def check_skinny_status(what: str = "skinny_gemm") -> None:
    """As check_status for the narrow projection, whose status word is a device variable (cleared when read)."""
    if not _status_checks[0]:
        return
    code = C.c_int(0)
    check(lib().rb2_skinny_gemm_status(C.byref(code), 1), "skinny_gemm_status")
    if code.value:
        raise DeviceStatusError(what, code.value)


def _current_stream(t):
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


class LaunchProfiler:
    """Device time of every library kernel launch between start() and read(), measured with
    CUDA events recorded on the launching stream."""

    def __init__(self, capacity: int = 4096):
        self.capacity = capacity

    def start(self):
        check(lib().rb2_profile_enable(self.capacity), "profile_enable")

    def read(self):
        lib().rb2_profile_disable()
        stride = 64
        names = C.create_string_buffer(self.capacity * stride)
        ms = (C.c_float * self.capacity)()
        n = lib().rb2_profile_read(self.capacity, names, stride, ms)
        if n < 0:
            check(ECUDA, "profile_read")
        raw = names.raw
        out = [(raw[i * stride:(i + 1) * stride].split(b"\0", 1)[0].decode(), float(ms[i])) for i in range(n)]
        return out, int(lib().rb2_profile_dropped())


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()
