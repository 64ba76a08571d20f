"""The fused channel half of a block (spx_block_channel_forward):
h_out = h + layer(RMSNorm(h)).update, against the oracle's RMSNorm feeding the
layer, at both combine paths, with K padding and with the MXFP8 lane."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.mixer_ref import rms_norm
from spalmer_b200 import B200ChannelBlock, MicroExpertsConfig
from tests.helpers import bf16_bits, from_bits, mxfp8_config, mxfp8_experts, set_mxfp8_lanes

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
    with torch.no_grad():
        h_out, out = block(h.to(DEV))
        # the reference order, unfused: RMSNorm (oracle, bit-exact to the reference's), layer, add
        x_bits = rms_norm(bf16_bits(h).reshape(-1, config.d_model), bf16_bits(block.channel_norm.weight.cpu()),
                          block.channel_norm.eps)
        ref = block.channel_mixer(from_bits(x_bits, DEV).reshape(batch, seq, -1))
    torch.cuda.synchronize()
    assert block.channel_mixer.device_status() == 0
    # the residual add in the combine is exactly bf16(h + update)
    assert torch.equal(h_out, (h.to(DEV).float() + out.update.float()).to(torch.bfloat16))
    # the fused RMSNorm feeds the same rows: same routing and update, bar rows whose
    # rsqrt sum of squares rounds to the neighbouring BF16 value
    same_rows = (out.update == ref.update).all(dim=-1).float().mean().item()
    assert same_rows > 0.99, same_rows
    ids_same = (out.metrics["expert_ids"] == ref.metrics["expert_ids"]).all(dim=-1).float().mean().item()
    assert ids_same > 0.99, ids_same
    diff = (out.update.float() - ref.update.float()).abs()
    assert (diff <= 1e-2 + 2e-2 * ref.update.float().abs()).float().mean().item() > 0.999
