"""MXFP8 restatement for the promoted-expert lane (test infrastructure only).

The reference's MXFP8 expert matmul (mESmaC/spalmer src/spalmer/experts/
native.py:91-140) quantises both operands row-wise along K in blocks of 32
(``MXTensor.to_mx(v, float8_e4m3fn, 32, ScaleCalculationMode.RCEIL)``) and
multiplies them with a block-scaled tensor-core GEMM whose result is cast to
BF16.  torchao (which implements ``to_mx``) is not a declared dependency of
the reference and is not installed here, so this module restates the
published algorithm (OCP Microscaling Formats v1.0, with the RCEIL scale rule
that cuBLAS documents for block quantisation):

* per block of 32 values: ``descale = amax / 448`` (float32 division);
  ``e = ceil(log2(descale))`` clamped to [-127, 127]; the E8M0 scale byte is
  ``e + 127``; blocks whose byte is 0 (amax below 448 * 2^-127, including
  all-zero blocks) use a multiplier of 1;
* elements: ``clamp(v * 2^-e, -448, 448)`` rounded to E4M3 (FN variant,
  round to nearest even);
* dequantised value: ``e4m3 * 2^(byte - 127)``.

Parity for this lane is unpinned beyond the reference's own bound (relative
error < 0.15 against FP32 math on the BF16 masters, tests/experts/
test_native_precision.py:27-79): ``ceil(log2(.))`` is computed exactly here
from the float's bits, while torchao evaluates log2 in float, which can round
the other way when descale lies within an ulp of a power of two.
"""

from __future__ import annotations

import numpy as np

from oracle.bf16 import bf16_bits_to_f32

E4M3_MAX = 448.0
BLOCK = 32


def ceil_log2_exact(v: np.ndarray) -> np.ndarray:
    """Exact ceil(log2(v)) for positive finite float32 v (int32)."""

    v = np.asarray(v, dtype=np.float32)
    m, e = np.frexp(v.astype(np.float64))  # v = m * 2^e, m in [0.5, 1)
    # ceil(log2(v)) = e - 1 when v is a power of two (m == 0.5), else e
    return np.where(m == 0.5, e - 1, e).astype(np.int32)


def scale_bytes(amax: np.ndarray) -> np.ndarray:
    """E8M0 scale bytes (uint8) for block maxima (float32, >= 0)."""

    amax = np.asarray(amax, dtype=np.float32)
    descale = (amax / np.float32(E4M3_MAX)).astype(np.float32)
    out = np.zeros(descale.shape, dtype=np.int32)
    pos = descale > 0
    e = np.zeros(descale.shape, dtype=np.int32)
    e[pos] = ceil_log2_exact(descale[pos])
    e = np.clip(e, -127, 127)
    out[pos] = e[pos] + 127
    out[~pos] = 0
    return out.astype(np.uint8)


def _e4m3_table() -> np.ndarray:
    """float value of every E4M3FN byte (NaN for 0x7F / 0xFF)."""

    b = np.arange(256, dtype=np.int32)
    sign = np.where(b & 0x80, -1.0, 1.0)
    exp = (b >> 3) & 0xF
    man = b & 0x7
    val = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1 + man / 8.0) * 2.0 ** (exp - 7))
    val = sign * val
    val[(b & 0x7F) == 0x7F] = np.nan
    return val.astype(np.float32)


E4M3_VALUES = _e4m3_table()
_POS_SORTED = np.sort(E4M3_VALUES[:0x7F])  # non-negative finite magnitudes, ascending


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """Round float32 to E4M3FN bytes, nearest even; |x| <= 448 expected."""

    x = np.asarray(x, dtype=np.float32)
    mag = np.abs(x).astype(np.float64)
    grid = _POS_SORTED.astype(np.float64)
    idx = np.searchsorted(grid, mag)  # first grid >= mag
    idx = np.clip(idx, 1, len(grid) - 1)
    lo, hi = grid[idx - 1], grid[idx]
    pick_hi = (mag - lo) > (hi - mag)
    tie = (mag - lo) == (hi - mag)
    # even mantissa = even code (codes are ascending with magnitude)
    pick_hi = pick_hi | (tie & ((idx % 2) == 0))
    code = np.where(pick_hi, idx, idx - 1)
    code = np.where(mag <= 0, 0, code)
    code = np.where(mag >= grid[-1], len(grid) - 1, code)
    return (code | np.where(np.signbit(x), 0x80, 0)).astype(np.uint8)


def quantize_rows(x_f32: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Row-wise MXFP8 along the last axis (length multiple of 32).

    Returns ``(e4m3 bytes [..., K], scale bytes [..., K/32])``.
    """

    x = np.asarray(x_f32, dtype=np.float32)
    K = x.shape[-1]
    if K % BLOCK:
        raise ValueError("last dimension must be a multiple of 32")
    blocks = x.reshape(*x.shape[:-1], K // BLOCK, BLOCK)
    amax = np.abs(blocks).max(axis=-1)
    sb = scale_bytes(amax)
    e = sb.astype(np.int32) - 127
    mult = np.where(sb == 0, 1.0, np.ldexp(1.0, -e)).astype(np.float32)
    scaled = np.clip(blocks * mult[..., None], -E4M3_MAX, E4M3_MAX).astype(np.float32)
    return f32_to_e4m3(scaled).reshape(x.shape), sb


def dequantize_rows(q: np.ndarray, sb: np.ndarray) -> np.ndarray:
    vals = E4M3_VALUES[q].reshape(*q.shape[:-1], q.shape[-1] // BLOCK, BLOCK)
    scale = np.ldexp(np.float32(1.0), sb.astype(np.int32) - 127).astype(np.float32)
    return (vals * scale[..., None]).reshape(q.shape).astype(np.float32)


def mxfp8_matmul_bits(a_bits: np.ndarray, b_rows_bits: np.ndarray) -> np.ndarray:
    """``bf16(deq(mx(a)) @ deq(mx(b_rows)).T)``: native.py:113-140 without the 128-padding
    (zero padding of M/N/K changes no real element).  BF16 inputs as bits, BF16 bits out."""

    from oracle.bf16 import f32_to_bf16_bits

    a = bf16_bits_to_f32(a_bits)
    b = bf16_bits_to_f32(b_rows_bits)
    qa, sa = quantize_rows(a)
    qb, sbb = quantize_rows(b)
    return f32_to_bf16_bits(dequantize_rows(qa, sa) @ dequantize_rows(qb, sbb).T)
