"""C-ABI boundary checks that need no GPU: the library loads, exports every declared symbol,
sizes workspaces and rejects bad arguments before touching the device."""
import ctypes as C
import os
import re

import pytest

from recant_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    with open(os.path.join(ROOT, "include", "recant_b200.h")) as f:
        return re.findall(r"RB2_API\s+[\w\s\*]+?\b(rb2_\w+)\s*\(", f.read())


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_symbols()
    assert len(names) >= 9
    lib = L.lib()
    for n in names:
        assert hasattr(lib, n), n
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"
    assert set(L.SIGNATURES) <= set(names)


def test_version_string():
    assert b"sm_100a" in L.lib().rb2_version()


def test_gdn_workspace_size_scales_with_problem():
    lib = L.lib()
    small = lib.rb2_gdn_workspace_size(1, 1024, 1, 4, 8, 128, 128, L.F32, L.GDN_EXACT)
    big = lib.rb2_gdn_workspace_size(4, 4096, 4, 16, 32, 128, 128, L.F32, L.GDN_EXACT)
    assert 0 < small < big
    # cu_seqlens form: B == 1 with N sequences
    assert lib.rb2_gdn_workspace_size(1, 5000, 7, 16, 32, 128, 128, L.F32, L.GDN_EXACT) > 0


@pytest.mark.parametrize("Hk,Hv,path", [(16, 32, L.GDN_FAST), (32, 32, L.GDN_FAST), (2, 32, L.GDN_FAST),
                                        (4, 8, L.GDN_EXACT)])
def test_gdn_workspace_split_sums_to_total(Hk, Hv, path):
    lib = L.lib()
    dt = L.BF16 if path == L.GDN_FAST else L.F32
    total = lib.rb2_gdn_workspace_size(4, 4096, 4, Hk, Hv, 128, 128, dt, path)
    saved, scratch = C.c_size_t(0), C.c_size_t(0)
    assert lib.rb2_gdn_workspace_split(4, 4096, 4, Hk, Hv, 128, 128, dt, path, C.byref(saved),
                                       C.byref(scratch)) == L.OK
    assert saved.value + scratch.value == total and saved.value > 0
    if path == L.GDN_FAST:
        # scratch holds dS (32 KB) and dV' (16 KB) per (chunk, head) for the chunk bound
        # tokens / 64 + n_seqs; the GQA group sums of dq / dk stay in the kernel's tensor memory
        n_ch = (4 * 4096 // 64 + 4) * Hv
        per_ch = n_ch * (32768 + 16384)
        assert per_ch <= scratch.value <= per_ch + 4096
    else:
        assert scratch.value == 0
    assert lib.rb2_gdn_workspace_split(4, 4096, 4, Hk, Hv, 128, 128, dt, path, None, None) == L.EINVAL


@pytest.mark.parametrize("dk", [16, 64, 256])
def test_gdn_rejects_unsupported_head_dim(dk):
    lib = L.lib()
    st = lib.rb2_gdn_fwd(None, None, None, None, None, None, None, 1, 64, 1, 1, 1, dk, dk, L.F32, 0, 1.0,
                         None, None, C.c_void_p(256), 1 << 30, None)
    assert st == L.EUNSUPPORTED
    assert b"128" in lib.rb2_last_error()


def test_gdn_rejects_bad_group_and_dtype():
    lib = L.lib()
    st = lib.rb2_gdn_fwd(None, None, None, None, None, None, None, 1, 64, 1, 3, 4, 128, 128, L.F32, 0, 1.0,
                         None, None, C.c_void_p(256), 1 << 30, None)
    assert st == L.EINVAL and b"multiple" in lib.rb2_last_error()
    st = lib.rb2_gdn_fwd(None, None, None, None, None, None, None, 1, 64, 1, 1, 1, 128, 128, 7, 0, 1.0,
                         None, None, C.c_void_p(256), 1 << 30, None)
    assert st == L.EINVAL


def test_gdn_rejects_small_workspace_before_launch():
    lib = L.lib()
    p = C.c_void_p(4096)
    st = lib.rb2_gdn_fwd(p, p, p, p, p, None, None, 1, 64, 1, 1, 1, 128, 128, L.F32, L.GDN_EXACT, 1.0,
                         p, None, p, 16, None)
    assert st == L.EWORKSPACE


def test_quantize_rejects_bad_shapes():
    lib = L.lib()
    p = C.c_void_p(4096)
    assert lib.rb2_nvfp4_quantize(p, 4, 24, L.BF16, 1, 0, 0, p, p, None, p, p, 256, None) == L.EINVAL
    assert lib.rb2_nvfp4_quantize(p, 0, 32, L.BF16, 1, 0, 0, p, p, None, p, p, 256, None) == L.EINVAL
    assert lib.rb2_nvfp4_quantize(p, 4, 32, 5, 1, 0, 0, p, p, None, p, p, 256, None) == L.EINVAL
    assert lib.rb2_nvfp4_quantize(C.c_void_p(4100), 4, 32, L.BF16, 1, 0, 0, p, p, None, p, p, 256, None) == L.EINVAL


def test_ops_refuse_cpu_tensors():
    import torch
    from recant_b200 import gdn_b200, quantize_fast
    x = torch.zeros(1, 64, 1, 128)
    with pytest.raises(ValueError):
        gdn_b200(x, x, x, torch.zeros(1, 64, 1), torch.zeros(1, 64, 1))
    with pytest.raises(ValueError):
        quantize_fast(torch.zeros(4, 32))


def test_registry_mirror():
    from recant_b200 import gdn as G, nvfp4 as N
    assert G.get_gdn_backend() == "b200" and "b200" in G.GDN_BACKENDS
    with pytest.raises(KeyError):
        G.set_gdn_backend("nope")
    assert N.get_gemm_backend() == "b200"
    with pytest.raises(KeyError):
        N.set_gemm_backend("nope")


def test_gdn_fast_path_rejects_misaligned_pointers():
    lib = L.lib()
    ok, bad = C.c_void_p(1 << 20), C.c_void_p((1 << 20) + 2)
    st = lib.rb2_gdn_fwd(bad, ok, ok, ok, ok, None, None, 1, 64, 1, 1, 1, 128, 128, L.BF16, L.GDN_FAST, 1.0,
                         ok, ok, ok, 1 << 40, None)
    assert st == L.EINVAL and b"aligned" in lib.rb2_last_error()


def test_gemv_dispatch_bound_fits_the_kernel_and_larger_shapes_are_refused():
    """gemm_b200 sends A of at most GEMV_MAX_M rows to rb2_nvfp4_gemv only while A, dequantized with
    4 floats of padding per 32 (K + K/8 per row), plus the kernel's 272-float lookup tables fit its
    200 KB of shared memory; the C entry refuses anything larger before touching the device."""
    from recant_b200 import nvfp4 as N
    assert 4 * (256 + 16 + N.GEMV_MAX_ELEMS) <= 200 * 1024
    m, k = N.GEMV_MAX_M, 16384
    assert m * (k + k // 8) > N.GEMV_MAX_ELEMS          # the dispatch keeps this shape on the tile GEMM
    lib = L.lib()
    fake = 1 << 20                                       # never dereferenced: refused before any launch
    st = lib.rb2_nvfp4_gemv(fake, fake, fake, fake, fake, fake, m, 256, k, fake, L.F32, None)
    assert st != 0 and "shared memory" in lib.rb2_last_error().decode()


def test_quantizer_index_tables_follow_from_the_e2m1_grid():
    """The quantize kernel picks e2m1 indices from packed 4-bit tables keyed by
    ceil(bits(a) / 2^21): round-to-nearest counts the midpoints strictly below a, stochastic
    rounding takes the first grid point not below a (at least 1). Rebuild both tables from the grid
    and the key rule, and check them against the constants in the kernel source."""
    import struct

    import numpy as np
    with open(os.path.join(ROOT, "recant_b200", "csrc", "nvfp4_quant.cu")) as f:
        src = f.read()
    grid = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    mids = [(a + b) / 2 for a, b in zip(grid, grid[1:])]

    def bits(x):
        return struct.unpack("<I", struct.pack("<f", x))[0]

    def key(x):
        return (bits(x) + 0x1FFFFF) >> 21
    # every decision point sits on a multiple of 2^21 in the bit pattern, so key order = value order
    assert all(bits(p) % (1 << 21) == 0 for p in mids + grid[1:])
    rn = [sum(key(p) < 500 + k for p in mids) for k in range(19)]
    lo = sum(v << (4 * k) for k, v in enumerate(rn[:16]))
    hi = sum(v << (4 * (k - 16)) for k, v in enumerate(rn[16:], start=16))
    assert f"0x{lo:X}ull" in src and f"0x{hi:X}u" in src, (hex(lo), hex(hi))
    sr = [max(sum(key(p) < 504 + k for p in grid[:7]), 1) for k in range(15)]
    packed = sum(v << (4 * k) for k, v in enumerate(sr))
    assert f"0x{packed:X}ull" in src, hex(packed)
    # and the tables reproduce the reference's rules on every float32 in [0, 6] near a decision point
    for p in mids + grid:
        for x in np.nextafter(np.float32(p), np.float32([-1, 7])).tolist() + [p]:
            a = min(float(np.float32(x)), 6.0)
            if a < 0:
                continue
            k_rn = min(max(key(a), 500), 518) - 500
            assert rn[k_rn] == sum(a > m for m in mids)
            k_sr = min(max(key(a), 504), 518) - 504
            assert sr[k_sr] == max(sum(a > g for g in grid[:7]), 1)


def test_lora_wgrad_workspace_and_argument_checks():
    """rb2_lora_wgrad: the workspace holds the status word, the tiles' counters and the per-split
    partials (growing with N); bad ranks, strides, alignment and short workspaces are refused
    before any CUDA call."""
    lib = L.lib()
    assert lib.rb2_lora_wgrad_workspace_size(0, 4096, 16) == 256
    small = lib.rb2_lora_wgrad_workspace_size(16384, 4096, 16)
    big = lib.rb2_lora_wgrad_workspace_size(16384, 8192, 16)
    assert 256 < small < big
    p, ws = C.c_void_p(4096), C.c_void_p(1 << 20)
    args = dict(ldd=256, ldh=16, M=128, N=256, R=16)

    def call(ws_bytes=1 << 30, **kw):
        a = {**args, **kw}
        return lib.rb2_lora_wgrad(p, a["ldd"], p, a["ldh"], a["M"], a["N"], a["R"], 1.0, p, a["R"], 1, ws, ws_bytes,
                                  None)

    assert call(R=0) == L.EINVAL and b"rank" in lib.rb2_last_error()
    assert call(R=65) == L.EINVAL
    assert call(ldd=250) == L.EINVAL and b"strides" in lib.rb2_last_error()
    assert call(ws_bytes=16) == L.EINVAL and b"workspace" in lib.rb2_last_error()
    assert lib.rb2_lora_wgrad(C.c_void_p(4100), 256, p, 16, 128, 256, 16, 1.0, p, 16, 1, ws, 1 << 30,
                              None) == L.EINVAL


def test_lora_up_argument_checks():
    """rb2_lora_up refuses ranks outside [1, 128], unknown rounding modes and a short workspace before
    any CUDA call."""
    lib = L.lib()
    assert lib.rb2_lora_up_workspace_size() >= 4
    p, ws = C.c_void_p(4096), C.c_void_p(1 << 20)

    def call(r=16, mode=0, ws_bytes=256):
        return lib.rb2_lora_up(p, 256, p, 16, p, 16, 128, 256, r, 2.0, mode, p, 256, ws, ws_bytes, None)

    assert call(r=0) == L.EINVAL and b"rank" in lib.rb2_last_error()
    assert call(r=129) == L.EINVAL
    assert call(mode=2) == L.EINVAL and b"mode" in lib.rb2_last_error()
    assert call(ws_bytes=8) == L.EINVAL and b"workspace" in lib.rb2_last_error()
