"""NVFP4 restatement for the ("nvfp4", "nvfp4") expert pair (test infrastructure only).

The reference's NVFP4 expert matmul (mESmaC/spalmer src/spalmer/experts/
native.py:205-262, used by ``native_expert_matmul`` at native.py:324-326)
pads K to a multiple of 32 and N to a multiple of 16, packs both operands with
torchao's ``NVFP4Tensor.to_nvfp4(v, per_tensor_scale=per_tensor_amax_to_scale
(amax(|v|)))`` and multiplies them with ``_addmm_nvfp4_dispatch``.  torchao is
not installed here (nor declared by the reference), so this module restates
its published NVFP4 recipe:

* per-tensor scale ``pts = amax / (448 * 6)`` (float32);
* per block of 16 consecutive K elements: ``s = e4m3_rn(clamp((block_amax / 6)
  / pts, 2^-6, 448))`` (UE4M3 scale byte), elements ``e2m1_rn(clamp(v / (pts *
  s), -6, 6))`` on the grid {0, 0.5, 1, 1.5, 2, 3, 4, 6} with ties to the even
  code, packed two per byte (even element in the low nibble);
* product: ``bf16((deq(a) @ deq(b).T) * (pts_a * pts_b))`` with float32
  accumulation, the per-tensor factor applied once before the BF16 rounding.

Parity for this lane is unpinned: no golden vectors of the reference's NVFP4
path exist (it needs torchao and an NVFP4 GPU), and whether torchao applies the
per-tensor factor before or after its BF16 rounding is not visible from the
reference.  The anchor is the reference's own bound: relative error < 0.30
against float32 math on the BF16 inputs (tests/experts/test_native_precision.py
cases ("nvfp4", "nvfp4", 0.30)).  An all-zero operand (amax 0, where the
restated formula divides by zero) quantises to zeros.
"""

from __future__ import annotations

import numpy as np

from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits
from oracle.mxfp8 import E4M3_VALUES, f32_to_e4m3

BLOCK = 16
TENSOR_DIV = np.float32(448.0 * 6.0)
SCALE_MIN = np.float32(2.0 ** -6)
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def e2m1_codes(x: np.ndarray) -> np.ndarray:
    """Round float32 (|x| <= 6) to E2M1 codes (sign in bit 3), nearest even."""

    x = np.asarray(x, dtype=np.float32)
    m = np.abs(x)
    code = np.select(
        [m <= 0.25, m < 0.75, m <= 1.25, m < 1.75, m <= 2.5, m < 3.5, m <= 5.0],
        [0, 1, 2, 3, 4, 5, 6], default=7).astype(np.uint8)
    return code | np.where(np.signbit(x), 8, 0).astype(np.uint8)


def e2m1_values(codes: np.ndarray) -> np.ndarray:
    codes = np.asarray(codes, dtype=np.uint8)
    v = E2M1_VALUES[codes & 7]
    return np.where(codes & 8, -v, v).astype(np.float32)


def padded_k(cols: int) -> int:
    return -(-cols // 256) * 256


def quantize_rows(x_f32: np.ndarray, amax: np.float32 | None = None):
    """NVFP4 of a matrix [rows, cols] with one per-tensor scale.

    Returns ``(codes [rows, kp] uint8, scale bytes [rows, kp/16] uint8, amax)``
    with kp = cols rounded up to 256 (zero columns beyond cols).
    """

    x = np.asarray(x_f32, dtype=np.float32)
    rows, cols = x.shape
    kp = padded_k(cols)
    xp = np.zeros((rows, kp), dtype=np.float32)
    xp[:, :cols] = x
    if amax is None:
        amax = np.float32(np.abs(x).max()) if x.size else np.float32(0.0)
    pts = np.float32(np.float32(amax) / TENSOR_DIV)
    if not pts > 0:
        return np.zeros((rows, kp), np.uint8), np.zeros((rows, kp // BLOCK), np.uint8), np.float32(amax)
    blocks = xp.reshape(rows, kp // BLOCK, BLOCK)
    bamax = np.abs(blocks).max(axis=-1).astype(np.float32)
    s = ((bamax / np.float32(6.0)).astype(np.float32) / pts).astype(np.float32)
    s = np.clip(s, SCALE_MIN, np.float32(448.0)).astype(np.float32)
    sb = f32_to_e4m3(s)
    total = (pts * E4M3_VALUES[sb]).astype(np.float32)
    data = np.clip((blocks / total[..., None]).astype(np.float32), -6.0, 6.0).astype(np.float32)
    return e2m1_codes(data).reshape(rows, kp), sb, np.float32(amax)


def pack_codes(codes: np.ndarray) -> np.ndarray:
    """Two codes per byte, the even element in the low nibble."""

    c = np.asarray(codes, dtype=np.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def dequantize_rows(codes: np.ndarray, sb: np.ndarray) -> np.ndarray:
    """Block-scaled values (without the per-tensor scale), float32."""

    v = e2m1_values(codes)
    rows, kp = v.shape
    return (v.reshape(rows, kp // BLOCK, BLOCK) * E4M3_VALUES[sb][..., None]).reshape(rows, kp).astype(np.float32)


def nvfp4_matmul_bits(a_bits: np.ndarray, b_rows_bits: np.ndarray) -> np.ndarray:
    """``native_nvfp4_linear`` forward (native.py:224-262): ``a @ b_rows.T`` with
    both operands in NVFP4; BF16 bits in and out."""

    a = bf16_bits_to_f32(a_bits)
    b = bf16_bits_to_f32(b_rows_bits)
    qa, sa, amax_a = quantize_rows(a)
    qb, sbb, amax_b = quantize_rows(b)
    acc = dequantize_rows(qa, sa) @ dequantize_rows(qb, sbb).T
    alpha = np.float32(np.float32(amax_a / TENSOR_DIV) * np.float32(amax_b / TENSOR_DIV))
    return f32_to_bf16_bits((acc.astype(np.float32) * alpha).astype(np.float32))
