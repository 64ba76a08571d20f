"""Training through the layer: gradients of the native backward (spx_layer_backward
plus library GEMMs for the weight gradients) against the reference's own
gradients (golden fixtures) and against the autograd oracle on the same
routing, at both batch classes."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import mixer_autograd as MA
from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig
from tests.helpers import build_mixer, from_bits
from tests.test_backward_oracle import CASES, load_backward_case, relnorm

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
# BF16 gradients summed in different orders (and, where a router logit rounds
# differently on the GPU, a token routed elsewhere): relative L2 error bound.
GRAD_RTOL = 3e-2


def train_step(mixer, x: torch.Tensor, d_update: torch.Tensor, d_aux: float, d_scores=None):
    mixer.zero_grad(set_to_none=True)
    xg = x.detach().clone().requires_grad_(True)
    out = mixer(xg)
    outs = [out.update, out.auxiliary_loss]
    grads = [d_update, torch.tensor(d_aux, dtype=torch.bfloat16, device=x.device)]
    if d_scores is not None:
        outs.append(out.metrics["router_scores"])
        grads.append(d_scores)
    torch.autograd.backward(outs, grads)
    got = {"x": xg.grad}
    for name, p in mixer.named_parameters():
        if p.grad is not None:
            got[name] = p.grad
    return out, got


@pytest.mark.parametrize("name", CASES)
def test_gradients_match_reference(name):
    arrays, meta = load_backward_case(name)
    mixer = build_mixer(meta, DEV).train()
    batch, seq = meta["shape"]
    d = meta["config"]["d_model"]
    x = from_bits(arrays["x"], DEV).reshape(batch, seq, d)
    d_update = from_bits(arrays["d_update"], DEV).reshape(batch, seq, d)
    out, got = train_step(mixer, x, d_update, meta["d_aux"])
    ids = out.metrics["expert_ids"].reshape(-1, meta["config"]["active_experts"]).cpu().numpy()
    assert (ids == arrays["expert_ids"]).all(axis=1).mean() > 0.98  # routing as the reference's, bar rounding
    assert set(meta["grads"]) <= set(got)
    for key in meta["grads"]:
        want = from_bits(arrays["grad__" + key])
        assert relnorm(got[key].cpu(), want) < GRAD_RTOL, (key, relnorm(got[key].cpu(), want))
    assert relnorm(got["x"].reshape(-1, d).cpu(), from_bits(arrays["grad_x"])) < GRAD_RTOL


@pytest.mark.parametrize(
    "cfg,shape",
    [
        (dict(d_model=256, num_experts=200, expert_inter_dim=64, shared_inter_dim=256, active_experts=8), (2, 1024)),
        (dict(d_model=128, num_experts=200, expert_inter_dim=32, shared_inter_dim=0, active_experts=4), (1, 192)),
        (dict(d_model=64, num_experts=24, expert_inter_dim=80, shared_inter_dim=64, active_experts=3,
              router_score_transform="identity"), (2, 300)),
    ],
    ids=["m10_shape", "decode_no_shared", "identity_odd_inter"],
)
def test_gradients_match_oracle_on_same_routing(cfg, shape):
    config = MicroExpertsConfig(**cfg)
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).to(DEV).train()
    batch, seq = shape
    g = torch.Generator().manual_seed(11)
    x = torch.randn(batch, seq, config.d_model, generator=g).to(torch.bfloat16)
    d_update = (0.05 * torch.randn(batch, seq, config.d_model, generator=g)).to(torch.bfloat16)
    d_scores = (0.01 * torch.randn(batch, seq, config.num_experts, generator=g)).to(torch.bfloat16)
    out, got = train_step(mixer, x.to(DEV), d_update.to(DEV), 0.5, d_scores.to(DEV))
    k = config.active_experts
    ids = out.metrics["expert_ids"].reshape(-1, k).cpu()
    sd = {name: p.detach().cpu() for name, p in mixer.named_parameters()}
    params = {name: sd[name] for name in MA.PARAM_NAMES if name in sd}
    want = MA.gradients(params, x.reshape(-1, config.d_model), k, d_update.reshape(-1, config.d_model), 0.5,
                        d_scores=d_scores.reshape(-1, config.num_experts), ids=ids,
                        identity_scores=config.router_score_transform == "identity")
    for key, w in want.items():
        gk = got[key].reshape(w.shape).cpu()
        assert relnorm(gk, w) < GRAD_RTOL, (key, relnorm(gk, w))


def test_training_refuses_mxfp8_experts():
    from spalmer_b200.native import NativeExpertPrecisionError
    from tests.helpers import mxfp8_config, mxfp8_experts, set_mxfp8_lanes

    config = mxfp8_config(d_model=128, num_experts=32, expert_inter_dim=64, active_experts=4)
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).to(DEV).train()
    set_mxfp8_lanes(mixer, mxfp8_experts(config.num_experts, 0.25))
    x = torch.randn(1, 64, 128, device=DEV).to(torch.bfloat16)
    with pytest.raises(NativeExpertPrecisionError):
        mixer(x)
    with torch.no_grad():
        mixer(x)  # inference still runs both lanes


def test_swiglu_backward_rows_against_torch_fp32():
    """spx_swiglu_backward_rows (the shared expert's SwiGLU backward in the
    training step) against a plain PyTorch FP32 statement of the same
    derivatives, on unit and non-unit row weights."""

    import torch.nn.functional as F

    from spalmer_b200 import _lib

    lib = _lib.load()
    T, S = 257, 96
    g = torch.Generator().manual_seed(7)
    gate, up, dh = (torch.randn(T, S, generator=g).to(torch.bfloat16).to(DEV) for _ in range(3))
    w = (torch.rand(T, generator=g) + 0.5).to(torch.bfloat16).to(DEV)
    gate_up = torch.cat([gate, up], 1).contiguous()
    h = torch.empty(T, S, dtype=torch.bfloat16, device=DEV)
    dgu = torch.empty(T, 2 * S, dtype=torch.bfloat16, device=DEV)
    dw = torch.empty(T, dtype=torch.float32, device=DEV)
    order = torch.arange(T, dtype=torch.int32, device=DEV).flip(0).contiguous()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    assert lib.spx_swiglu_backward_rows(gate_up.data_ptr(), 2 * S, S, dh.data_ptr(), S, w.data_ptr(),
                                        order.data_ptr(), T, S, S, h.data_ptr(), dgu.data_ptr(), dw.data_ptr(),
                                        stream) == 0
    torch.cuda.synchronize()
    gf, uf, dhf, wf = gate.float(), up.float(), dh.float(), w.float()[:, None]
    sig = torch.sigmoid(gf)
    hf = F.silu(gf) * uf
    dhw = dhf * wf
    want_dgate = dhw * uf * sig * (1 + gf * (1 - sig))
    want_dup = dhw * F.silu(gf)
    # the hidden rows come out times their weight (the down projection's weight gradient takes h * w)
    for got, want in ((h, hf * wf), (dgu[:, :S], want_dgate), (dgu[:, S:], want_dup)):
        torch.testing.assert_close(got.float(), want, rtol=2e-2, atol=1e-2)
    torch.testing.assert_close(dw.flip(0), (dhf * hf).sum(1), rtol=2e-2, atol=1e-2 * S)
    # refused on the host before any launch: chunk not a multiple of 8
    assert lib.spx_swiglu_backward_rows(gate_up.data_ptr(), 2 * S, 4, dh.data_ptr(), S, w.data_ptr(),
                                        order.data_ptr(), T, S, S, h.data_ptr(), dgu.data_ptr(), dw.data_ptr(),
                                        stream) != 0
