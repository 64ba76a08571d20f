"""The fused channel half of a block (spx_block_channel_forward):
h_out = h + layer(RMSNorm(h)).update.  The fused call equals, bit for bit,
the unfused layer applied to the device RMSNorm's rows (spx_rmsnorm_rows), at
both combine paths, with K padding and with the MXFP8 lane; the device
RMSNorm equals the oracle's (bit-exact to the reference's) on every row
except where the float sum of squares, summed in another order, moves
bf16(rsqrt(...)) by one BF16 step, and those rows equal the oracle's rows
recomputed with that neighbouring step."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits
from oracle.mixer_ref import rms_norm
from spalmer_b200 import B200ChannelBlock, MicroExpertsConfig, rms_norm as device_rms_norm
from tests.helpers import bf16_bits, mxfp8_config, mxfp8_experts, set_mxfp8_lanes

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

CASES = {
    # fused combine (> 256 tokens), 100M-preset widths
    "m100_widths": (dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768,
                         active_experts=8), (1, 1024), False),
    # separate combine (decode-sized), d not a multiple of 64 (K padding of the normalised rows)
    "decode_padded": (dict(d_model=96, num_experts=40, expert_inter_dim=32, shared_inter_dim=64,
                           active_experts=4), (1, 64), False),
    # MXFP8 lane quantises the normalised rows
    "mxfp8": (dict(d_model=256, num_experts=64, expert_inter_dim=64, shared_inter_dim=256,
                   active_experts=8), (2, 256), True),
}


def _norm_given_r(h_bits: np.ndarray, w_bits: np.ndarray, r: np.ndarray) -> np.ndarray:
    """The two BF16 products of RMSNorm given each row's BF16 factor r."""

    x = f32_to_bf16_bits((bf16_bits_to_f32(h_bits) * r[:, None]).astype(np.float32))
    return f32_to_bf16_bits((bf16_bits_to_f32(x) * bf16_bits_to_f32(w_bits)[None, :]).astype(np.float32))


def _bf16_step(r: np.ndarray, up: bool) -> np.ndarray:
    bits = f32_to_bf16_bits(r.astype(np.float32)).astype(np.int32) + (1 if up else -1)
    return bf16_bits_to_f32(bits.astype(np.uint16))


def _check_norm_rows(got: np.ndarray, h_bits: np.ndarray, w_bits: np.ndarray, eps: float) -> float:
    want = rms_norm(h_bits, w_bits, eps)
    diff_rows = np.nonzero((got != want).any(axis=1))[0]
    if diff_rows.size:
        h = bf16_bits_to_f32(h_bits[diff_rows])
        var = np.square(h, dtype=np.float32).mean(axis=-1, dtype=np.float32)
        r = bf16_bits_to_f32(f32_to_bf16_bits((np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)))
        up = _norm_given_r(h_bits[diff_rows], w_bits, _bf16_step(r, True))
        down = _norm_given_r(h_bits[diff_rows], w_bits, _bf16_step(r, False))
        ok = (got[diff_rows] == up).all(axis=1) | (got[diff_rows] == down).all(axis=1)
        assert ok.all(), f"rows {diff_rows[~ok][:8]} differ beyond one step of r"
    return diff_rows.size


@pytest.mark.parametrize("name", CASES)
def test_block_matches_norm_then_layer_then_residual(name):
    cfg, (batch, seq), mx = CASES[name]
    config = mxfp8_config(**cfg) if mx else MicroExpertsConfig(**cfg)
    torch.manual_seed(0)
    block = B200ChannelBlock(config).to(torch.bfloat16).to(DEV).eval()
    if mx:
        set_mxfp8_lanes(block.channel_mixer, mxfp8_experts(config.num_experts, 0.25))
    g = torch.Generator().manual_seed(3)
    with torch.no_grad():
        block.channel_norm.weight.copy_(1.0 + 0.1 * torch.randn(config.d_model, generator=g))
    h = (torch.randn(batch, seq, config.d_model, generator=g) * 2.0).to(torch.bfloat16)
    eps = block.channel_norm.eps
    with torch.no_grad():
        h_out, out = block(h.to(DEV))
        # unfused, in the reference's order: RMSNorm, layer, add
        xn = device_rms_norm(h.to(DEV), block.channel_norm.weight, eps)
        ref = block.channel_mixer(xn)
    torch.cuda.synchronize()
    assert block.channel_mixer.device_status() == 0
    # the fused call is the unfused layer on the same rows, bit for bit
    assert torch.equal(out.metrics["expert_ids"], ref.metrics["expert_ids"])
    assert torch.equal(out.metrics["routing_weights"], ref.metrics["routing_weights"])
    assert torch.equal(out.update, ref.update)
    # the residual add in the combine is exactly bf16(h + update)
    assert torch.equal(h_out, (h.to(DEV).float() + out.update.float()).to(torch.bfloat16))
    # the device RMSNorm against the oracle's
    moved = _check_norm_rows(bf16_bits(xn).reshape(-1, config.d_model), bf16_bits(h).reshape(-1, config.d_model),
                             bf16_bits(block.channel_norm.weight.cpu()), eps)
    assert moved <= max(2, batch * seq // 100), moved


@pytest.mark.parametrize("rows,d", [(0, 64), (1, 8), (37, 96), (4096, 1024), (3, 4096)])
def test_rmsnorm_rows_matches_oracle(rows, d):
    """spx_rmsnorm_rows alone: empty input, one row, ragged row counts, and
    rows wider than the register path (d > 2048)."""

    g = torch.Generator().manual_seed(rows + d)
    h = (torch.randn(rows, d, generator=g) * 3.0).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    got = device_rms_norm(h.to(DEV), w.to(DEV), 1e-6)
    torch.cuda.synchronize()
    assert got.shape == h.shape
    if rows:
        moved = _check_norm_rows(bf16_bits(got), bf16_bits(h), bf16_bits(w), 1e-6)
        assert moved <= max(2, rows // 100), moved
