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


def _with_workspace(x, rht, sr, seed):
    lib = L.lib()
    m, k = x.shape
    c, s, b, g = _outputs(m, k, x.device)
    wsb = lib.rb2_nvfp4_quantize_workspace_size(m, k)
    ws = torch.empty(wsb, dtype=torch.uint8, device=x.device)
    st = lib.rb2_nvfp4_quantize(x.data_ptr(), m, k, L.BF16, rht, sr, seed, c.data_ptr(), s.data_ptr(), b.data_ptr(),
                                g.data_ptr(), ws.data_ptr(), wsb, torch.cuda.current_stream().cuda_stream)
    L.check(st, "nvfp4_quantize")
    return c, s, b, g


def _no_alloc(x, rht, sr, seed):
    lib = L.lib()
    m, k = x.shape
    c, s, b, g = _outputs(m, k, x.device)
    st = lib.rb2_nvfp4_quantize_noalloc(x.data_ptr(), m, k, L.BF16, rht, sr, seed, c.data_ptr(), s.data_ptr(),
                                        b.data_ptr(), g.data_ptr(), torch.cuda.current_stream().cuda_stream)
    L.check(st, "nvfp4_quantize_noalloc")
    return c, s, b, g


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
