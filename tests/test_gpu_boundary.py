"""The lower seams of the drop-in on the GPU: ``SurpriseRouter.forward``
(experts/router.py:40-56) through ``spx_router_forward`` and
``MicroExpertBank.execute_routing`` (experts/bank.py:593-646) through
``spx_gather_rows`` / ``spx_experts_forward`` / ``spx_combine``.

Router: bit-identical to the scores the fused layer computes, within the BF16
tolerance of the reference's own scores (the GEMM's accumulation order
differs), gradients within tolerance of an FP32 restatement.  Bank: within
the BF16 tolerance (rtol 2e-2, atol 1e-2) of the reference's own outputs on
arbitrary pairs (ragged, empty tokens, a token with 30 pairs, grouped and loop
executors, a restricted resident set) and of the oracle, BF16 and MXFP8 lanes.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import mixer_ref as R
from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig
from tests.conftest import LAYER_CASES, load_layer_case
from tests.helpers import bf16_bits, build_mixer, from_bits, mxfp8_config, mxfp8_experts, oracle_params
from tests.test_bank_oracle import load_bank, seeded_mixer
from tests.test_gpu_parity import assert_close_bf16

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("name", LAYER_CASES)
def test_router_forward_matches_layer_and_reference(name):
    arrays, meta = load_layer_case(name)
    mixer = build_mixer(meta, DEV)
    batch, seq = meta["shape"]
    x = from_bits(arrays["x"], DEV).reshape(batch, seq, -1)
    with torch.no_grad():
        scores = mixer.router(x)
        layer = mixer(x)
    torch.cuda.synchronize()
    assert scores.shape == (batch, seq, meta["config"]["num_experts"]) and scores.dtype == torch.bfloat16
    assert torch.equal(scores, layer.metrics["router_scores"])
    assert_close_bf16(bf16_bits(scores).reshape(arrays["router_scores"].shape), arrays["router_scores"])


def test_router_forward_ragged_shapes_and_errors():
    arrays, meta = load_layer_case("bias_resident")
    mixer = build_mixer(meta, DEV)
    x = from_bits(arrays["x"], DEV)
    for rows in (1, 7, 129, 256, 257):
        with torch.no_grad():
            got = mixer.router(x[:rows])
            want = mixer.router(x)[:rows]
        assert torch.equal(got, want), rows
    with pytest.raises(ValueError):
        mixer.router(x[:, :-1])
    with pytest.raises(RuntimeError):
        mixer.router(x.float())


def test_router_forward_gradients():
    arrays, meta = load_layer_case("bias_resident")
    mixer = build_mixer(meta, DEV)
    router = mixer.router
    x = from_bits(arrays["x"], DEV).requires_grad_(True)
    g = torch.randn(x.shape[0], meta["config"]["num_experts"], generator=torch.Generator().manual_seed(5))
    g = (0.1 * g).to(torch.bfloat16).to(DEV)
    scores = router(x)
    torch.autograd.backward(scores, g)
    # FP32 restatement of softplus(F.linear(x, W, b)) and its gradients
    xf = x.detach().float().requires_grad_(True)
    wf = router.proj.weight.detach().float().requires_grad_(True)
    bf = router.proj.bias.detach().float().requires_grad_(True)
    ref = torch.nn.functional.softplus(xf @ wf.t() + bf)
    torch.autograd.backward(ref, g.float())
    for got, want in ((x.grad, xf.grad), (router.proj.weight.grad, wf.grad), (router.proj.bias.grad, bf.grad)):
        err = (got.float() - want).norm() / want.norm()
        assert float(err) < 2e-2


@pytest.mark.parametrize("case", ["grouped", "loop", "resident"])
def test_execute_routing_matches_reference(case):
    arrays, meta = load_bank()
    execution = meta["cases"][case]["execution"]
    mixer = seeded_mixer(meta, execution, DEV)
    x = from_bits(arrays["x"], DEV)
    tok = torch.from_numpy(arrays[f"{case}__token_index"].astype(np.int64)).to(DEV)
    ids = torch.from_numpy(arrays[f"{case}__expert_index"].astype(np.int64)).to(DEV)
    w = from_bits(arrays[f"{case}__weights"], DEV)
    resident = arrays.get(f"{case}__resident_ids")
    res_t = None if resident is None else torch.from_numpy(resident.astype(np.int64)).to(DEV)
    with torch.no_grad():
        out = mixer.experts.execute_routing(x, tok, ids, w, None, res_t)
        again = mixer.experts.execute_routing(x, tok, ids, w, None, res_t)
    torch.cuda.synchronize()
    assert out.shape == (x.shape[0], x.shape[1]) and out.dtype == torch.bfloat16
    assert torch.equal(out, again)
    got = bf16_bits(out)
    assert_close_bf16(got, arrays[f"{case}__update"])
    params = oracle_params(mixer.cpu())
    want = R.execute_routing(arrays["x"], arrays[f"{case}__token_index"], arrays[f"{case}__expert_index"],
                             arrays[f"{case}__weights"], params.gate, params.up, params.down,
                             execution=execution, resident_ids=resident)
    assert_close_bf16(got, want)
    assert not np.any(got[48:])  # tokens without pairs stay zero


def test_execute_routing_mixer_layout_matches_layer_routed_part():
    """The mixer's own pairs (p = t*k + j) through the bank seam equal the
    oracle's routed update given the reference's ids and weights."""

    arrays, meta = load_layer_case("m10_slice")
    mixer = build_mixer(meta, DEV)
    k = meta["config"]["active_experts"]
    ids = arrays["expert_ids"].astype(np.int64)
    T = ids.shape[0]
    x = from_bits(arrays["x"], DEV)
    tok = torch.arange(T, device=DEV).repeat_interleave(k)
    with torch.no_grad():
        out = mixer.experts.execute_routing(x, tok, torch.from_numpy(ids.reshape(-1)).to(DEV),
                                            from_bits(arrays["routing_weights"].reshape(-1), DEV))
    params = oracle_params(mixer)
    want, _, _ = R.grouped_experts(arrays["x"], ids, arrays["routing_weights"], params.gate, params.up, params.down)
    assert_close_bf16(bf16_bits(out), want)


def test_execute_routing_mxfp8_lane_and_empty():
    cfg = dict(d_model=256, num_experts=64, expert_inter_dim=64, shared_inter_dim=0, active_experts=4)
    config = mxfp8_config(**cfg)
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(DEV)
    lane = mxfp8_experts(64, 0.5)
    promoted = torch.from_numpy(~lane).to(DEV)  # promoted experts run BF16, the rest MXFP8
    rng = np.random.default_rng(3)
    N, P = 96, 500
    tok = rng.integers(0, N - 10, size=P).astype(np.int64)
    ids = rng.integers(0, 64, size=P).astype(np.int64)
    w = torch.from_numpy(rng.uniform(0.1, 1.0, size=P).astype(np.float32)).to(torch.bfloat16)
    x = torch.randn(N, 256, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    with torch.no_grad():
        out = mixer.experts.execute_routing(x.to(DEV), torch.from_numpy(tok).to(DEV), torch.from_numpy(ids).to(DEV),
                                            w.to(DEV), promoted)
        empty = mixer.experts.execute_routing(x.to(DEV), torch.zeros(0, dtype=torch.long, device=DEV),
                                              torch.zeros(0, dtype=torch.long, device=DEV),
                                              torch.zeros(0, dtype=torch.bfloat16, device=DEV), promoted)
    params = oracle_params(mixer)
    want = R.execute_routing(bf16_bits(x), tok, ids, bf16_bits(w), params.gate, params.up, params.down, lane_mx=lane)
    assert_close_bf16(bf16_bits(out), want)
    assert not torch.any(empty)
    with pytest.raises(ValueError):
        mixer.experts.execute_routing(x.to(DEV), torch.zeros(3, dtype=torch.long, device=DEV),
                                      torch.zeros(2, dtype=torch.long, device=DEV),
                                      torch.zeros(3, dtype=torch.bfloat16, device=DEV))
