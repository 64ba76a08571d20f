"""bfloat16 helpers for the numpy oracle (test infrastructure only).

numpy has no bfloat16 dtype, so BF16 tensors are carried as ``uint16`` bit
patterns and arithmetic is done in float32/float64 with an explicit
round-to-nearest-even back to BF16 at every point where the reference's
PyTorch CPU kernels produce a BF16 tensor.  The rounding rule is the one of
``c10::BFloat16`` (round half to even on the upper 16 bits; NaN becomes the
canonical quiet NaN ``0x7FC0``).
"""

from __future__ import annotations

import numpy as np

BF16_NAN = np.uint16(0x7FC0)


def f32_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """Round float32 values to BF16 (RNE) and return the ``uint16`` bit patterns."""

    a = np.ascontiguousarray(values, dtype=np.float32)
    u = a.view(np.uint32)
    bias = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    with np.errstate(over="ignore"):
        out = ((u + bias) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = BF16_NAN
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen BF16 bit patterns to float32 (exact)."""

    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_bf16(values: np.ndarray) -> np.ndarray:
    """float32 -> nearest BF16 value, returned as float32."""

    return bf16_bits_to_f32(f32_to_bf16_bits(values))


def f64_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """float64 -> float32 (RNE) -> BF16 (RNE), the conversion PyTorch applies to doubles."""

    return f32_to_bf16_bits(np.asarray(values, dtype=np.float64).astype(np.float32))
