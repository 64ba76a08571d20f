"""CPU checks of the MXFP8 restatement (oracle/mxfp8.py).

torchao (which holds the reference's MXFP8 arithmetic, experts/native.py:91-110)
is not installed, so the restatement is pinned piecewise: the E4M3 element cast
against torch's own ``float8_e4m3fn`` conversion, the E8M0 encoding against
``float8_e8m0fnu``, the RCEIL scale rule on hand-worked cases, and the
end-to-end error against the reference's own bound (relative error < 0.15
versus FP32 math, tests/experts/test_native_precision.py:27-79).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import mxfp8
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits


def test_e4m3_cast_matches_torch_including_ties_and_subnormals():
    rng = np.random.default_rng(0)
    grid = mxfp8._POS_SORTED.astype(np.float64)
    mids = ((grid[1:] + grid[:-1]) / 2).astype(np.float32)
    vals = np.concatenate(
        [rng.standard_normal(50000).astype(np.float32) * s for s in (1e-3, 1e-2, 0.1, 1.0, 10.0, 100.0)]
        + [mids, -mids, grid.astype(np.float32), -grid.astype(np.float32),
           np.nextafter(mids, np.float32(np.inf)), np.nextafter(mids, np.float32(0)),
           np.array([0.0, -0.0, 448.0, -448.0], dtype=np.float32)]
    )
    vals = np.clip(vals, -448, 448).astype(np.float32)
    ours = mxfp8.f32_to_e4m3(vals)
    ref = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(ours, ref)


def test_e8m0_bias_matches_torch():
    e = np.arange(-127, 128)
    ref = torch.from_numpy(np.ldexp(1.0, e).astype(np.float32)).to(torch.float8_e8m0fnu).view(torch.uint8).numpy()
    np.testing.assert_array_equal(ref, e + 127)


@pytest.mark.parametrize(
    "amax,byte",
    [
        (0.0, 0),                       # all-zero block: multiplier 1
        (448.0, 127),                   # descale exactly 1
        (448.0 * 2.0 ** 5, 132),        # exact power of two: no round-up
        (np.nextafter(np.float32(448.0), np.float32(1e9)), 128),  # just above: RCEIL rounds up
        (1.0, 127 - 8),                 # 1/448 in (2^-9, 2^-8]: ceil -> -8
        (448.0 * 2.0 ** -127, 0),       # smallest scale
        (1e-40, 0),                     # below the scale range: clamped to -127
    ],
)
def test_rceil_scale_rule(amax, byte):
    assert int(mxfp8.scale_bytes(np.array([amax], dtype=np.float32))[0]) == byte


def test_quantised_elements_stay_within_e4m3_range_and_error():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((64, 256)) * np.exp(rng.uniform(-8, 8, (64, 1)))).astype(np.float32)
    x = bf16_bits_to_f32(f32_to_bf16_bits(x))
    q, sb = mxfp8.quantize_rows(x)
    assert q.shape == x.shape and sb.shape == (64, 8)
    assert not np.any((q & 0x7F) == 0x7F)  # no NaN codes
    deq = mxfp8.dequantize_rows(q, sb)
    # per-block: amax maps into (224, 448] so normal elements carry <= 2^-4 relative error
    blocks = np.abs(x).reshape(64, 8, 32)
    err = np.abs(deq - x).reshape(64, 8, 32)
    scale = np.ldexp(1.0, sb.astype(np.int64) - 127)[..., None]
    assert np.all(err <= np.maximum(blocks * 2.0 ** -4, scale * 2.0 ** -10) + 1e-30)


def test_mxfp8_matmul_meets_the_reference_bound():
    """Shapes and bound of test_native_precision.py:27-79 (forward, relative error < 0.15)."""

    gen = torch.Generator().manual_seed(1204)
    a = torch.randn((7, 37), generator=gen).to(torch.bfloat16)
    w = torch.randn((23, 37), generator=gen).to(torch.bfloat16)
    pad = lambda t: torch.nn.functional.pad(t, (0, 64 - 37))  # noqa: E731 - K padded with zeros
    a_bits = pad(a).view(torch.int16).numpy().view(np.uint16)
    w_bits = pad(w).view(torch.int16).numpy().view(np.uint16)
    out = bf16_bits_to_f32(mxfp8.mxfp8_matmul_bits(a_bits, w_bits))
    ref = (a.float() @ w.float().t()).numpy()
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel < 0.15, rel
    assert rel < 0.05  # MXFP8 with 1x32 blocks is far inside the bound
