"""The quantization telemetry restated in the oracle
(``MicroExpertBank.quantization_error``, experts/bank.py:526-592, with
``native_weight_reconstruction_error``, experts/native.py:391-417): properties
the reference's definition implies, checked on the CPU."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import mixer_ref as R
from oracle.bf16 import f32_to_bf16_bits


def _bits(x: np.ndarray) -> np.ndarray:
    return f32_to_bf16_bits(np.asarray(x, dtype=np.float32))


@pytest.mark.parametrize("fmt", ["mxfp8", "nvfp4"])
def test_zero_matrix_has_zero_error(fmt):
    assert R.reconstruction_error(np.zeros((8, 64), dtype=np.uint16), fmt) == 0.0


def test_mxfp8_exact_blocks_have_zero_error():
    """Blocks of E4M3 grid values whose amax is 448 times a power of two
    quantise without loss (scale = that power of two)."""

    rng = np.random.default_rng(0)
    grid = np.array([1.0, 0.5, 2.0, -3.0, 0.75, -1.25, 6.0, -10.0, 14.0, 0.125], dtype=np.float32)
    w = rng.choice(grid, size=(16, 96)).astype(np.float32)
    w[:, ::32] = 448.0  # every 32-value block reaches 448 x 2^-10 after the scaling below
    w *= np.float32(2.0 ** -10)
    assert R.reconstruction_error(_bits(w), "mxfp8") == 0.0


@pytest.mark.parametrize("fmt", ["mxfp8", "nvfp4"])
def test_error_is_invariant_under_power_of_two_scaling(fmt):
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((24, 128)) * 0.05).astype(np.float32)
    base = R.reconstruction_error(_bits(w), fmt)
    for k in (-3, 4):
        assert R.reconstruction_error(_bits(w * np.float32(2.0 ** k)), fmt) == base


def test_typical_magnitudes_and_format_order():
    rng = np.random.default_rng(2)
    w = _bits((rng.standard_normal((64, 256)) * 0.02).astype(np.float32))
    mx = R.reconstruction_error(w, "mxfp8")
    nv = R.reconstruction_error(w, "nvfp4")
    assert 1e-4 < mx < 1e-2  # 3 mantissa bits: relative MSE near 2^-8
    assert mx < nv < 0.2     # E2M1 is coarser


def test_ragged_k_matches_explicit_zero_padding():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((8, 40)) * 0.1).astype(np.float32)
    padded = np.zeros((8, 64), dtype=np.float32)
    padded[:, :40] = w
    for fmt in ("mxfp8", "nvfp4"):
        assert R.reconstruction_error(_bits(w), fmt) == R.reconstruction_error(_bits(padded), fmt)


def test_quantization_error_selects_and_averages():
    rng = np.random.default_rng(4)
    E, d, I = 6, 64, 32
    gate = _bits(rng.standard_normal((E, d, I)) * 0.05)
    up = _bits(rng.standard_normal((E, d, I)) * 0.05)
    down = _bits(rng.standard_normal((E, I, d)) * 0.05)
    ids = np.array([[1, 4], [4, 5]])
    got = R.quantization_error(ids, gate, up, down, "mxfp8")
    assert np.all(got[[0, 2, 3]] == 0.0) and np.all(got[[1, 4, 5]] > 0.0)
    e = 4
    parts = [R.reconstruction_error(np.ascontiguousarray(m[e].T), "mxfp8") for m in (gate, up, down)]
    assert got[e] == np.float32(np.float32(np.float32(parts[0] + parts[1]) + parts[2]) / np.float32(3.0))
    assert np.all(R.quantization_error(ids, gate, up, down, "bfloat16") == 0.0)
