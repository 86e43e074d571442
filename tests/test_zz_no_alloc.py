"""The allocation-free quantizer entry point (rb2_nvfp4_quantize_noalloc).

It exists for callers that cannot give the library device scratch: C/C++ embedders without a
device allocator, serving loops running with a frozen allocator, code where a cudaMalloc would
synchronise or exceed a memory cap. Its scratch word lives in a static device buffer instead.
This file is collected last so that a failure here comes after every other test has run; it must
pass both alone in a fresh process and after the rest of the suite.
"""
import pytest
import torch

from recant_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _outputs(m, k, device):
    return (torch.empty(m, k // 2, dtype=torch.uint8, device=device),
            torch.empty(m, k // 16, dtype=torch.uint8, device=device),
            torch.empty(-(-m // 128) * -(-(k // 16) // 4) * 512, dtype=torch.uint8, device=device),
            torch.empty(1, dtype=torch.float32, device=device))


_DT = {torch.bfloat16: L.BF16, torch.float32: L.F32}


def _with_workspace(x, rht, sr, seed, blocked=True):
    lib = L.lib()
    m, k = x.shape
    c, s, b, g = _outputs(m, k, x.device)
    wsb = lib.rb2_nvfp4_quantize_workspace_size(m, k)
    ws = torch.empty(wsb, dtype=torch.uint8, device=x.device)
    st = lib.rb2_nvfp4_quantize(x.data_ptr(), m, k, _DT[x.dtype], rht, sr, seed, c.data_ptr(), s.data_ptr(),
                                b.data_ptr() if blocked else None, g.data_ptr(), ws.data_ptr(), wsb,
                                torch.cuda.current_stream().cuda_stream)
    L.check(st, "nvfp4_quantize")
    return (c, s, b, g) if blocked else (c, s, g)


def _no_alloc(x, rht, sr, seed, blocked=True):
    lib = L.lib()
    m, k = x.shape
    c, s, b, g = _outputs(m, k, x.device)
    st = lib.rb2_nvfp4_quantize_noalloc(x.data_ptr(), m, k, _DT[x.dtype], rht, sr, seed, c.data_ptr(), s.data_ptr(),
                                        b.data_ptr() if blocked else None, g.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
    L.check(st, "nvfp4_quantize_noalloc")
    return (c, s, b, g) if blocked else (c, s, g)


@pytest.mark.parametrize("rht,sr", [(1, 0), (0, 0), (1, 1)])
def test_noalloc_matches_workspace_entry_point_twice(rht, sr):
    """Two calls in a row (different inputs, so the shared scratch must be cleared in between)
    give exactly what the workspace entry point gives; quantizer outputs are bit-exact."""
    gen = torch.Generator().manual_seed(17 + rht + 2 * sr)
    for call, (m, k) in enumerate(((300, 2048), (257, 6144))):
        x = (torch.randn(m, k, generator=gen) * (30.0 if call == 0 else 0.5)).to(torch.bfloat16).cuda()
        seed = 1234 + call
        ref = _with_workspace(x, rht, sr, seed)
        got = _no_alloc(x, rht, sr, seed)
        torch.cuda.synchronize()
        for a, b in zip(ref, got):
            assert torch.equal(a, b)


@pytest.mark.parametrize("dtype,shapes,blocked", [
    (torch.bfloat16, ((8, 2048), (3, 512)), True),      # at most 2048 blocks: the one-CTA path
    (torch.float32, ((300, 2048), (5, 160)), True),     # f32 input, both paths
    (torch.bfloat16, ((257, 6144), (130, 64)), False),  # no blocked-scale output
])
def test_noalloc_small_f32_and_unblocked_twice(dtype, shapes, blocked):
    """The same comparison on the single-CTA path (which needs no scratch word), on f32 input and
    with scales_blocked = NULL; two calls in a row, each bit-exact with the workspace entry point."""
    gen = torch.Generator().manual_seed(41)
    for call, (m, k) in enumerate(shapes):
        x = (torch.randn(m, k, generator=gen) * (4.0 if call == 0 else 0.25)).to(dtype).cuda()
        ref = _with_workspace(x, 1, 0, 0, blocked)
        got = _no_alloc(x, 1, 0, 0, blocked)
        torch.cuda.synchronize()
        for a, b in zip(ref, got):
            assert torch.equal(a, b)
