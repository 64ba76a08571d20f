"""The NVFP4 restatement (oracle/nvfp4.py) on its own: the E2M1 grid and its
ties, the UE4M3 block-scale rule, zero padding, and the reference's own error
bound for the ("nvfp4", "nvfp4") pair (relative error < 0.30 against float32
math, mESmaC/spalmer tests/experts/test_native_precision.py)."""

from __future__ import annotations

import numpy as np

from oracle import nvfp4 as NV
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits


def test_e2m1_grid_and_ties():
    x = np.array([0, 0.25, 0.26, 0.5, 0.75, 1.0, 1.25, 1.3, 1.75, 2.5, 2.6, 3.5, 5.0, 5.1, 6.0, -0.75, -5.0, -0.1],
                 dtype=np.float32)
    want = [0, 0, 0.5, 0.5, 1.0, 1.0, 1.0, 1.5, 2.0, 2.0, 3.0, 4.0, 4.0, 6.0, 6.0, -1.0, -4.0, 0.0]
    np.testing.assert_array_equal(NV.e2m1_values(NV.e2m1_codes(x)), np.array(want, dtype=np.float32))
    assert NV.e2m1_codes(np.array([-0.1], np.float32))[0] == 8  # sign kept on a value rounding to zero


def test_block_scale_rule_and_padding():
    x = np.zeros((2, 40), dtype=np.float32)
    x[0, :16] = np.linspace(-3, 3, 16)
    x[1, 16:32] = 0.001
    codes, sb, amax = NV.quantize_rows(x)
    assert codes.shape == (2, 256) and sb.shape == (2, 16) and amax == np.float32(3.0)
    pts = np.float32(3.0) / np.float32(2688.0)
    # block 0 of row 0: amax 3 -> scale (3/6)/pts = 448 exactly
    assert sb[0, 0] == NV.f32_to_e4m3(np.array([448.0], np.float32))[0]
    # an all-zero block clamps its scale to 2^-6 and quantises to zero codes
    assert NV.E4M3_VALUES[sb[0, 5]] == np.float32(2.0 ** -6) and not codes[0, 80:96].any()
    deq = NV.dequantize_rows(codes, sb) * pts
    np.testing.assert_allclose(deq[0, :16], x[0, :16], atol=0.5 + 1e-6)  # half the widest grid gap (2 units of 0.5)
    np.testing.assert_array_equal(NV.pack_codes(np.array([[1, 2, 3, 4]], np.uint8)), [[0x21, 0x43]])
    zc, zs, za = NV.quantize_rows(np.zeros((3, 20), np.float32))
    assert za == 0 and not zc.any() and not zs.any()


def test_matmul_within_reference_bound():
    rng = np.random.default_rng(0)
    for m, n, k in [(64, 48, 96), (33, 16, 300), (128, 200, 512)]:
        a = f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
        b = f32_to_bf16_bits((0.02 * rng.standard_normal((n, k))).astype(np.float32))
        got = bf16_bits_to_f32(NV.nvfp4_matmul_bits(a, b))
        want = bf16_bits_to_f32(a) @ bf16_bits_to_f32(b).T
        rel = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert rel < 0.30, rel
        assert rel > 1e-3  # genuinely quantised
