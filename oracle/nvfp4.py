"""NVFP4 oracle in numpy -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates, bit for bit, the reference quantizer in recant/model/nvfp4.py:

* ``rht``            -- nvfp4.py:15-31  (per-16 sign flip, butterfly strides 1,2,4,8 as
                        (a+b, a-b), x0.25, cast back to the input dtype)
* ``quantize``       -- nvfp4.py:76-91  (global scale, per-16 e4m3 scales, RN codes with
                        ties toward zero, -0 code for small negatives, nibble pack)
* ``round_codes_sr`` -- nvfp4.py:59-71  (stochastic branch; numpy RNG, statistical only)
* ``to_blocked``     -- nvfp4.py:112-119 (128x4 blocked scale swizzle of torch._scaled_mm)
* ``dequant`` / ``gemm_emulated`` -- nvfp4.py:45-57,108-110

All arithmetic is float32 with IEEE round-to-nearest (numpy float32 ops), matching torch's
CPU kernels, so codes, scales and the global scale are bit-exact with the reference.
"""
from __future__ import annotations

import numpy as np

BLOCK = 16
FP4_MAX = np.float32(6.0)
E4M3_MAX = np.float32(448.0)
FP4_GRID = np.array((0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0), dtype=np.float32)
# Decision midpoints between neighbouring e2m1 magnitudes; a value equal to a midpoint
# rounds DOWN (toward zero): torch.bucketize(right=False) counts boundaries strictly below.
MIDS = np.array((0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0), dtype=np.float32)
# torch.randint(0, 2, (16,), generator=manual_seed(1234)) * 2 - 1  (nvfp4.py:21)
SIGNS = np.array([1, 1, -1, 1, -1, -1, -1, 1, 1, 1, 1, 1, -1, -1, 1, -1], dtype=np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 (ties to even), returned as float32."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def _e4m3_table() -> np.ndarray:
    c = np.arange(127)                       # 127 = NaN in e4m3fn; 126 = 448
    e, m = c >> 3, c & 7
    return np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * 2.0 ** (e - 7.0))


E4M3_VALUES = _e4m3_table()                  # float64, increasing, exact


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """Non-negative float32 in [0, 448] -> e4m3fn byte, round to nearest even."""
    xd = np.asarray(x, dtype=np.float64)
    lo = np.clip(np.searchsorted(E4M3_VALUES, xd, side="right") - 1, 0, 126)
    hi = np.minimum(lo + 1, 126)
    vlo, vhi = E4M3_VALUES[lo], E4M3_VALUES[hi]
    mid = (vlo + vhi) / 2.0
    pick_hi = (xd > mid) | ((xd == mid) & (lo % 2 == 1))
    code = np.where(pick_hi & (hi != lo), hi, lo)
    return code.astype(np.uint8)


def e4m3_decode(code: np.ndarray) -> np.ndarray:
    c = np.asarray(code, dtype=np.uint8)
    mag = E4M3_VALUES[np.minimum(c & 0x7F, 126)].astype(np.float32)
    return np.where(c & 0x80, -mag, mag).astype(np.float32)


def rht(x: np.ndarray, dtype: str) -> np.ndarray:
    """16-point randomized Hadamard transform per row block (nvfp4.py:23-31).

    ``dtype`` is the tensor's dtype ('bf16' or 'f32'): the result is re-rounded to it.
    """
    m, k = x.shape
    g = k // BLOCK
    y = x.astype(np.float32).reshape(m, g, BLOCK) * SIGNS
    for s in (1, 2, 4, 8):
        y = y.reshape(m, g, BLOCK // (2 * s), 2, s)
        a, b = y[..., 0, :], y[..., 1, :]
        y = np.stack([a + b, a - b], axis=-2)
    y = (y.reshape(m, k) * np.float32(0.25)).astype(np.float32)
    return bf16_round(y) if dtype == "bf16" else y


def _scales(x: np.ndarray):
    m, k = x.shape
    amax = np.float32(np.abs(x).max()) if x.size else np.float32(0.0)
    s_g = np.float32(np.maximum(amax, np.float32(1e-30)) / np.float32(FP4_MAX * E4M3_MAX))
    xb = x.reshape(m, k // BLOCK, BLOCK)
    bmax = np.abs(xb).max(-1)
    s_b = np.minimum((bmax / FP4_MAX).astype(np.float32) / s_g, E4M3_MAX).astype(np.float32)
    s8 = e4m3_encode(s_b)
    sq = e4m3_decode(s8)
    denom = (np.where(sq == 0, np.float32(1.0), sq) * s_g).astype(np.float32)
    return xb, s8, denom, s_g


def round_codes_rn(q: np.ndarray) -> np.ndarray:
    a = np.minimum(np.abs(q), FP4_MAX)
    idx = (a[..., None] > MIDS).sum(-1)
    return (idx + 8 * (q < 0)).astype(np.uint8)


def round_codes_sr(q: np.ndarray, u: np.ndarray) -> np.ndarray:
    """Unbiased rounding to a neighbouring grid point (nvfp4.py:62-68); u ~ U[0,1)."""
    a = np.minimum(np.abs(q), FP4_MAX)
    hi = np.maximum((a[..., None] > FP4_GRID).sum(-1), 1)
    lo = hi - 1
    glo, ghi = FP4_GRID[lo], FP4_GRID[hi]
    p = ((a - glo) / (ghi - glo)).astype(np.float32)
    idx = np.where(u < p, hi, lo)
    return (idx + 8 * (q < 0)).astype(np.uint8)


def pack(codes: np.ndarray) -> np.ndarray:
    """Two 4-bit codes per byte, even element in the low nibble (nvfp4.py:73-74)."""
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)


def quantize(x: np.ndarray, stochastic: bool = False, rng=None):
    """x: float32 [M, K] (already RHT'd and re-rounded) -> (codes u8 [M,K/2], scales u8
    (e4m3 bytes) [M,K/16], gscale float32)."""
    assert x.ndim == 2 and x.shape[1] % BLOCK == 0, x.shape
    m, k = x.shape
    x = np.ascontiguousarray(x, dtype=np.float32)
    xb, s8, denom, s_g = _scales(x)
    q = (xb / denom[..., None]).astype(np.float32)
    if stochastic:
        rng = rng or np.random.default_rng(0)
        codes = round_codes_sr(q, rng.random(q.shape, dtype=np.float32))
    else:
        codes = round_codes_rn(q)
    return pack(codes.reshape(m, k)), s8, np.float32(s_g)


def quantize_activation(x: np.ndarray, dtype: str, use_rht: bool = True,
                        stochastic: bool = False, rng=None):
    """quantize(rht(x)) as nvfp4.quantize_activation's reference branch (nvfp4.py:144-149)."""
    return quantize(rht(x, dtype) if use_rht else np.asarray(x, np.float32), stochastic, rng)


def to_blocked(scales_u8: np.ndarray) -> np.ndarray:
    """[rows, cols] scale bytes -> flat 128x4-blocked swizzle (nvfp4.py:112-119)."""
    rows, cols = scales_u8.shape
    nrb, ncb = -(-rows // 128), -(-cols // 4)
    u = np.zeros((nrb * 128, ncb * 4), dtype=np.uint8)
    u[:rows, :cols] = scales_u8
    blocks = u.reshape(nrb, 128, ncb, 4).transpose(0, 2, 1, 3)
    return blocks.reshape(-1, 4, 32, 4).transpose(0, 2, 1, 3).reshape(-1).copy()


def unpack(codes: np.ndarray, k: int) -> np.ndarray:
    lo, hi = codes & 15, codes >> 4
    return np.stack([lo, hi], -1).reshape(codes.shape[0], k)


def dequant(codes: np.ndarray, scales_u8: np.ndarray, gscale, k: int) -> np.ndarray:
    """value = grid[c&7] * sign * (scale * gscale)  (nvfp4.py:45-57), float32."""
    c = unpack(codes, k)
    val = FP4_GRID[c & 7] * np.where(c & 8, np.float32(-1.0), np.float32(1.0))
    sc = (np.repeat(e4m3_decode(scales_u8), BLOCK, axis=-1) * np.float32(gscale)).astype(np.float32)
    return (val * sc).astype(np.float32)


def gemm_emulated(a, b) -> np.ndarray:
    """a, b: (codes, scales, gscale, (rows, k)) -> a . b^T in float32 (nvfp4.py:108-110): both
    operands dequantised to float32 and multiplied by torch's CPU float32 matmul with the second
    operand transposed, the same call the reference's emulated backend makes, so that the sums run
    in the same order."""
    import torch
    ka, kb = a[3][1], b[3][1]
    da = torch.from_numpy(np.ascontiguousarray(dequant(a[0], a[1], a[2], ka), dtype=np.float32))
    db = torch.from_numpy(np.ascontiguousarray(dequant(b[0], b[1], b[2], kb), dtype=np.float32))
    return (da @ db.t()).float().numpy()


def quantize_weight(w: np.ndarray, use_rht: bool = True):
    """fprop = Q(rht(W)), dgrad = Q(rht(W^T)), fp32 RHT with no re-rounding (nvfp4.py:101-106)."""
    n, k = w.shape
    wf = np.asarray(w, np.float32)
    fp = quantize(rht(wf, "f32") if use_rht else wf)
    wt = np.ascontiguousarray(wf.T)
    dg = quantize(rht(wt, "f32") if use_rht else wt)
    return (fp + ((n, k),)), (dg + ((k, n),))
