"""GPU parity of the MXFP8 lane (block-scaled tcgen05 GEMM) against the oracle.

Bit-exact: the quantiser (E4M3 values and E8M0 scale bytes).  Within BF16
rounding of the oracle: the dense MXFP8 matmul (both sides use the same
quantised operands; only the FP32 accumulation order differs).  Within the
layer contract (rtol 2e-2, atol 1e-2): layers whose experts run in MXFP8, in
BF16, or mixed, given identical router logits.  The reference's own bound
(relative error < 0.15 against FP32 math on the BF16 masters,
tests/experts/test_native_precision.py:27-79) is checked on its shapes.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import mixer_ref as R
from oracle import mxfp8 as MX
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits
from spalmer_b200 import B200MicroExpertChannelMixer
from spalmer_b200.native import mx_quantize_rows, mxfp8_mm_nt, native_expert_matmul
from tests.helpers import (bf16_bits, from_bits, mxfp8_config, mxfp8_experts, oracle_params, set_mxfp8_lanes,
                           torch_layer_update)

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
RTOL, ATOL = 2e-2, 1e-2


def _rows(shape, seed, spread=6.0):
    """BF16 rows with per-row magnitudes spread over e^+-spread, a zero block and tiny values."""

    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape) * np.exp(rng.uniform(-spread, spread, (shape[0], 1)))
    if shape[1] >= 64:
        x[0, :32] = 0.0
        x[1, 32:64] = 1e-39  # subnormal block
    return f32_to_bf16_bits(x.astype(np.float32))


@pytest.mark.parametrize("rows,cols", [(300, 768), (7, 32), (129, 160), (30000, 768)])
def test_quantize_rows_is_bit_exact(rows, cols):
    bits = _rows((rows, cols), seed=rows + cols)
    q, s = mx_quantize_rows(from_bits(bits, DEV))
    want_q, want_s = MX.quantize_rows(bf16_bits_to_f32(bits))
    assert np.array_equal(s.cpu().numpy(), want_s)
    assert np.array_equal(q.cpu().numpy(), want_q)


def _mm_close(got_bits, want_bits):
    a = bf16_bits_to_f32(got_bits).astype(np.float64)
    b = bf16_bits_to_f32(want_bits).astype(np.float64)
    tol = 1e-2 * np.abs(b) + 1e-3 * max(1.0, np.abs(b).max())
    bad = np.abs(a - b) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside; max |diff| {np.abs(a - b).max()}"


@pytest.mark.parametrize("m,n,k", [(7, 23, 37), (128, 128, 128), (300, 200, 768), (257, 130, 96), (1, 16, 32)])
def test_mxfp8_mm_nt_matches_oracle(m, n, k):
    a = _rows((m, k), seed=1, spread=2.0)
    b = _rows((n, k), seed=2, spread=2.0)
    got = bf16_bits(mxfp8_mm_nt(from_bits(a, DEV), from_bits(b, DEV)))
    kp = (k + 31) // 32 * 32
    pad = lambda v: np.pad(v, ((0, 0), (0, kp - k)))  # noqa: E731 - zero K padding, as the reference
    _mm_close(got, MX.mxfp8_matmul_bits(pad(a), pad(b)))


def test_reference_native_precision_bound():
    """test_native_precision.py:27-79 forward: relative error < 0.15 vs FP32 matmul."""

    gen = torch.Generator(device="cpu").manual_seed(1204)
    x = torch.randn((7, 37), generator=gen).to(device=DEV, dtype=torch.bfloat16)
    w = torch.randn((23, 37), generator=gen).to(device=DEV, dtype=torch.bfloat16)
    out = mxfp8_mm_nt(x, w)
    ref = x.float() @ w.float().t()
    rel = float((out.float() - ref).norm() / ref.norm().clamp_min(1e-12))
    assert rel < 0.15, rel
    # expert layout [in, out] (native_expert_matmul, experts/native.py:305-350)
    out2 = native_expert_matmul(x, w.t().contiguous(), weight_format="mxfp8", activation_format="mxfp8")
    assert torch.equal(out2, out)


LAYER_SHAPES = {
    "smoke": (dict(d_model=128, num_experts=200, expert_inter_dim=32, shared_inter_dim=128, active_experts=4), (2, 256)),
    "m100_slice": (dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768, active_experts=8),
                   (2, 1024)),
}


def _layer(name, fraction, seed=0):
    cfg_kw, (batch, seq) = LAYER_SHAPES[name]
    config = mxfp8_config(**cfg_kw)
    torch.manual_seed(seed)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(DEV)
    lane = mxfp8_experts(config.num_experts, fraction)
    set_mxfp8_lanes(mixer, lane)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(batch, seq, config.d_model, generator=gen).to(torch.bfloat16)
    return mixer, lane, bf16_bits(x).reshape(-1, config.d_model), batch, seq


@pytest.mark.parametrize("name", list(LAYER_SHAPES))
@pytest.mark.parametrize("fraction", [0.25, 1.0, 0.0])
def test_mxfp8_layer_matches_oracle_given_logits(name, fraction):
    mixer, lane, x_bits, batch, seq = _layer(name, fraction)
    params = oracle_params(mixer)
    k = mixer.config.active_experts
    logits = R.router_logits(x_bits, params.router_w, params.router_b)
    x = from_bits(x_bits, DEV).reshape(batch, seq, -1)
    with torch.no_grad():
        out = mixer(x, router_logits=from_bits(logits, DEV).reshape(batch, seq, -1))
    torch.cuda.synchronize()
    assert mixer.device_status() == 0
    want = R.mixer_forward(params, x_bits, k, logit_bits=logits, lane_mx=lane)
    assert np.array_equal(out.metrics["expert_ids"].cpu().numpy().reshape(-1, k), want["expert_ids"])
    assert np.array_equal(bf16_bits(out.metrics["routing_weights"]).reshape(-1, k), want["routing_weights"])
    got = bf16_bits_to_f32(bf16_bits(out.update).reshape(want["update"].shape)).astype(np.float64)
    ref = bf16_bits_to_f32(want["update"]).astype(np.float64)
    bad = np.abs(got - ref) > ATOL + RTOL * np.abs(ref)
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; max |diff| {np.abs(got - ref).max()}"
    if 0.0 < fraction < 1.0:
        # The lanes differ: the same layer run all-BF16 gives a different update.
        set_mxfp8_lanes(mixer, np.zeros_like(lane))
        with torch.no_grad():
            out_bf16 = mixer(x, router_logits=from_bits(logits, DEV).reshape(batch, seq, -1))
        assert not torch.equal(out_bf16.update, out.update)


def test_mxfp8_layer_full_size_sample_and_determinism():
    """100M shape, 25% of experts MXFP8: sampled rows vs the oracle, every row
    vs the FP32 torch restatement, bitwise-stable reruns."""

    config = mxfp8_config(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768, active_experts=8)
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(DEV)
    lane = mxfp8_experts(200, 0.25)
    set_mxfp8_lanes(mixer, lane)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(64, 1024, 768, generator=gen).to(torch.bfloat16)
    x_bits = bf16_bits(x).reshape(-1, 768)
    xd = x.to(DEV)
    with torch.no_grad():
        out = mixer(xd)
        again = mixer(xd)
    torch.cuda.synchronize()
    assert mixer.device_status() == 0
    assert torch.equal(out.update, again.update)
    k = 8
    ids = out.metrics["expert_ids"].cpu().numpy().reshape(-1, k)
    weights = bf16_bits(out.metrics["routing_weights"]).reshape(-1, k)
    params = oracle_params(mixer)
    rng = np.random.default_rng(5)
    sample = np.sort(rng.choice(ids.shape[0], size=256, replace=False))
    routed, _, _ = R.grouped_experts(x_bits[sample], ids[sample], weights[sample], params.gate, params.up,
                                     params.down, lane_mx=lane)
    shared = R.shared_swiglu(x_bits[sample], params.shared_gate, params.shared_up, params.shared_down)
    want = R.f32_to_bf16_bits(bf16_bits_to_f32(routed) + bf16_bits_to_f32(shared))
    got = bf16_bits_to_f32(bf16_bits(out.update).reshape(-1, 768)[sample]).astype(np.float64)
    ref = bf16_bits_to_f32(want).astype(np.float64)
    bad = np.abs(got - ref) > ATOL + RTOL * np.abs(ref)
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance"
    # every update row against the FP32 torch restatement on the device
    full = torch_layer_update(mixer, xd.reshape(-1, 768), out.metrics["expert_ids"].reshape(-1, k),
                              out.metrics["routing_weights"].reshape(-1, k), lane_mx=lane)
    got_all = bf16_bits_to_f32(bf16_bits(out.update).reshape(-1, 768)).astype(np.float64)
    ref_all = bf16_bits_to_f32(bf16_bits(full)).astype(np.float64)
    bad = np.abs(got_all - ref_all) > 1e-3 + RTOL * np.abs(ref_all)
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance (all rows)"
