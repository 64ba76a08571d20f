"""Decode-shaped batches (1-64 tokens per step) through the grouped expert
GEMVs (``gemv.cu``, used up to 1024 routed pairs): the layer update within the
BF16 tolerance (rtol 2e-2, atol 1e-2) of the oracle given the layer's own
routing, at the 100M widths (d=768, I=128, k=8), all-BF16 and with a seeded
10% of the experts in MXFP8; the GEMV and the tcgen05 paths agree on the same
tokens across the 1024-pair boundary; a 16-layer stack replayed as a CUDA
graph equals the eager stack bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import mixer_ref as R
from oracle.bf16 import bf16_bits_to_f32
from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig
from tests.helpers import bf16_bits, mxfp8_config, mxfp8_experts, oracle_params, set_mxfp8_lanes
from tests.test_gpu_parity import assert_close_bf16

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
CFG = dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768, active_experts=8)


def _mixer(mx_fraction: float, seed: int = 0):
    config = mxfp8_config(**CFG) if mx_fraction else MicroExpertsConfig(**CFG)
    torch.manual_seed(seed)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(DEV)
    lane = None
    if mx_fraction:
        lane = mxfp8_experts(config.num_experts, mx_fraction)
        set_mxfp8_lanes(mixer, lane)
    return mixer, lane


def _oracle_update(mixer, lane, x_bits, ids, w_bits):
    params = oracle_params(mixer)
    routed, _, _ = R.grouped_experts(x_bits, ids, w_bits, params.gate, params.up, params.down, lane_mx=lane)
    shared = R.shared_swiglu(x_bits, params.shared_gate, params.shared_up, params.shared_down)
    return R.f32_to_bf16_bits(bf16_bits_to_f32(routed) + bf16_bits_to_f32(shared))


@pytest.mark.parametrize("mx_fraction", [0.0, 0.1])
@pytest.mark.parametrize("tokens", [1, 8, 64, 128])
def test_decode_layer_matches_oracle(tokens, mx_fraction):
    mixer, lane = _mixer(mx_fraction)
    x = torch.randn(1, tokens, CFG["d_model"], generator=torch.Generator().manual_seed(10 + tokens))
    x = x.to(torch.bfloat16)
    with torch.no_grad():
        out = mixer(x.to(DEV))
        again = mixer(x.to(DEV))
    torch.cuda.synchronize()
    assert mixer.device_status() == 0
    assert torch.equal(out.update, again.update)
    k = CFG["active_experts"]
    ids = out.metrics["expert_ids"].cpu().numpy().reshape(-1, k)
    w_bits = bf16_bits(out.metrics["routing_weights"]).reshape(-1, k)
    want = _oracle_update(mixer, lane, bf16_bits(x).reshape(tokens, -1), ids, w_bits)
    assert_close_bf16(bf16_bits(out.update).reshape(want.shape), want)


@pytest.mark.parametrize("mx_fraction", [0.0, 0.25])
def test_gemv_and_tensor_core_paths_agree(mx_fraction):
    """128 tokens (1024 pairs: GEMVs) and the same tokens plus one (1032 pairs:
    tcgen05 GEMMs): the first 128 rows agree within the BF16 tolerance."""

    mixer, _ = _mixer(mx_fraction)
    x = torch.randn(1, 129, CFG["d_model"], generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).to(DEV)
    with torch.no_grad():
        small = mixer(x[:, :128].contiguous())
        large = mixer(x)
    torch.cuda.synchronize()
    assert mixer.device_status() == 0
    assert torch.equal(small.metrics["expert_ids"], large.metrics["expert_ids"][:, :128])
    assert_close_bf16(bf16_bits(small.update), bf16_bits(large.update[:, :128].contiguous()))


def test_decode_stack_graph_replay_matches_eager():
    layers = [_mixer(0.1, seed=s)[0] for s in range(4)]
    x = torch.randn(1, 64, CFG["d_model"], generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).to(DEV)

    def stack(h):
        for m in layers:
            h = h + m(h).update
        return h

    with torch.inference_mode():
        want = stack(x)
        static_x = x.clone()
        for _ in range(2):
            stack(static_x)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = stack(static_x)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, want)
        del graph
    for m in layers:
        assert m.device_status() == 0


def test_decode_skewed_expert_many_rows():
    """All 64 tokens on the same 8 experts (rows beyond one 16-row pass)."""

    config = MicroExpertsConfig(**CFG, router_bias=True)
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(DEV)
    with torch.no_grad():
        bias = torch.full((200,), 30.0)
        bias[:8] = -30.0  # softplus scores: these eight are always the least surprised
        mixer.router.proj.bias.copy_(bias.to(torch.bfloat16))
    x = torch.randn(1, 64, CFG["d_model"], generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    with torch.no_grad():
        out = mixer(x.to(DEV))
    torch.cuda.synchronize()
    ids = out.metrics["expert_ids"].cpu().numpy().reshape(-1, 8)
    assert set(np.unique(ids).tolist()) == set(range(8))
    w_bits = bf16_bits(out.metrics["routing_weights"]).reshape(-1, 8)
    want = _oracle_update(mixer, None, bf16_bits(x).reshape(64, -1), ids, w_bits)
    assert_close_bf16(bf16_bits(out.update).reshape(want.shape), want)
