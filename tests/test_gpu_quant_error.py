"""Quantization telemetry on the device: ``spx_expert_quant_error`` (every
expert's reconstruction error, computed when the masters change) against the
oracle's restatement of ``native_weight_reconstruction_error``
(experts/native.py:391-417), and the forward's ``expert_quantization_error``
metric (``MicroExpertBank.quantization_error``, experts/bank.py:526-566): the
error of each selected expert, zero elsewhere, for MXFP8 and NVFP4 expert
weights, through the small (one-CTA) and the large dispatch; zeros for BF16
weights.  Float tolerance: relative 1e-5 (the device sums in double, the
oracle exactly; the reference in float32)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import mixer_ref as R
from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig
from tests.helpers import bf16_bits, mxfp8_experts, set_mxfp8_lanes

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
SHAPE = dict(d_model=256, num_experts=48, expert_inter_dim=96, shared_inter_dim=256, active_experts=4)


def _mixer(fmt: str):
    kw = dict(SHAPE)
    if fmt != "bfloat16":
        kw.update(expert_weight_format=fmt, expert_activation_format=fmt, expert_promotion_format="bfloat16")
    config = MicroExpertsConfig(**kw)
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).to(DEV).eval()
    if fmt != "bfloat16":
        set_mxfp8_lanes(mixer, mxfp8_experts(config.num_experts, 0.25))
    return mixer


def _masters(mixer):
    sd = mixer.state_dict()
    return tuple(bf16_bits(sd[f"experts.{n}_proj"]) for n in ("gate", "up", "down"))


@pytest.mark.parametrize("fmt", ["mxfp8", "nvfp4"])
def test_every_expert_error_matches_oracle(fmt):
    mixer = _mixer(fmt)
    got = mixer._quant_error(DEV).cpu().numpy()
    want = R.expert_reconstruction_errors(*_masters(mixer), fmt)
    assert np.all(want > 0)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=0)


@pytest.mark.parametrize("tokens", [64, 4096], ids=["small_dispatch", "large_dispatch"])
@pytest.mark.parametrize("fmt", ["mxfp8", "nvfp4", "bfloat16"])
def test_forward_metric_reports_selected_experts(fmt, tokens):
    mixer = _mixer(fmt)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(1, tokens, SHAPE["d_model"], generator=g).to(torch.bfloat16).to(DEV)
    with torch.no_grad():
        out = mixer(x)
    torch.cuda.synchronize()
    assert mixer.device_status() == 0
    got = out.metrics["expert_quantization_error"].cpu().numpy()
    ids = out.metrics["expert_ids"].cpu().numpy()
    want = R.quantization_error(ids, *_masters(mixer), fmt)
    selected = np.zeros(SHAPE["num_experts"], dtype=bool)
    selected[np.unique(ids)] = True
    assert np.all(got[~selected] == 0.0)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=0)


def test_error_follows_weight_updates():
    mixer = _mixer("mxfp8")
    before = mixer._quant_error(DEV).clone()
    with torch.no_grad():
        mixer.experts.gate_proj[3].mul_(0.0)
    after = mixer._quant_error(DEV).cpu().numpy()
    want = R.expert_reconstruction_errors(*_masters(mixer), "mxfp8")
    np.testing.assert_allclose(after, want, rtol=1e-5, atol=0)
    assert after[3] != before[3].item()
