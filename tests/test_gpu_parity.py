"""GPU parity: libspx (through its C ABI) against the reference fixtures and the oracle.

Bit-exact: softplus scores, expert ids and their order, routing weights,
dispatch permutation, counts and telemetry scalars, given identical router
logits.  Within the BF16 tolerance of the contract (rtol 2e-2, atol 1e-2,
FP32 accumulators): the layer update and the auxiliary loss.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import mixer_ref as R
from oracle.bf16 import bf16_bits_to_f32
from oracle.topk import topk_least
from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig, dispatch, route
from spalmer_b200.experts import softplus_table
from tests.conftest import LAYER_CASES, load_layer_case
from tests.golden.topk_cases import TOPK_CASES, generate_scores
from tests.helpers import bf16_bits, build_mixer, from_bits, oracle_params, resident_mask, torch_layer_update

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 1e-2
DEV = torch.device("cuda", 0)


def assert_close_bf16(got_bits, want_bits, rtol=RTOL, atol=ATOL):
    a = bf16_bits_to_f32(got_bits).astype(np.float64)
    b = bf16_bits_to_f32(want_bits).astype(np.float64)
    bad = np.abs(a - b) > atol + rtol * np.abs(b)
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; max |diff| {np.abs(a - b).max()}"


def test_softplus_table_is_exact_for_every_bf16_input():
    table = softplus_table(DEV).cpu().numpy().view(np.uint16)
    want = R.softplus_lut()
    x = bf16_bits_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    finite = ~np.isnan(x)
    assert np.array_equal(table[finite], want[finite])
    assert np.all(np.isnan(bf16_bits_to_f32(table[~finite])))


@pytest.mark.parametrize("name", LAYER_CASES)
def test_route_from_reference_logits_is_bit_exact(name):
    arrays, meta = load_layer_case(name)
    cfg = meta["config"]
    mask = resident_mask(meta)
    scores, ids, weights = route(
        from_bits(arrays["logits"], DEV), cfg["active_experts"], transform=cfg["router_score_transform"],
        resident_mask=None if mask is None else torch.from_numpy(mask),
    )
    torch.cuda.synchronize()
    assert np.array_equal(bf16_bits(scores), arrays["router_scores"])
    assert np.array_equal(ids.cpu().numpy(), arrays["expert_ids"].astype(np.int64))
    assert np.array_equal(bf16_bits(weights), arrays["routing_weights"])


@pytest.mark.parametrize("tiled", [False, True], ids=["rows_kernel", "select_ties_kernels"])
@pytest.mark.parametrize("case", TOPK_CASES, ids=[c["name"] for c in TOPK_CASES])
def test_route_tie_order_matches_reference_topk(case, golden_topk, tiled):
    """Small batches take the warp-per-row route kernel; batches above 4096
    rows (the fixture tiled) take route_select + route_ties."""

    scores_bits, mask = generate_scores(case)
    reps = -(-4097 // scores_bits.shape[0]) if tiled else 1
    logits = from_bits(np.tile(scores_bits, (reps, 1)), DEV)  # identity transform: logits are the scores
    for k in case["ks"]:
        _, ids, _ = route(logits, k, transform="identity",
                          resident_mask=None if mask is None else torch.from_numpy(mask))
        got = ids.cpu().numpy()
        want = np.tile(golden_topk[f"{case['name']}__k{k}"].astype(np.int64), (reps, 1))
        rows = np.nonzero((got != want).any(axis=1))[0]
        assert rows.size == 0, f"k={k}: {rows.size} rows differ, first {rows[:5]}"


def _zipf_ids(tokens, k, experts, seed):
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, experts + 1) ** 1.1
    p /= p.sum()
    perm = rng.permutation(experts)
    out = np.empty((tokens, k), dtype=np.int64)
    for t in range(tokens):
        out[t] = perm[rng.choice(experts, size=k, replace=False, p=p)]
    return out


@pytest.mark.parametrize("tokens,k,experts", [(4096, 8, 200), (1000, 4, 200), (333, 2, 6), (50000, 8, 200)])
def test_dispatch_is_stable_argsort(tokens, k, experts):
    ids = _zipf_ids(tokens, k, experts, seed=tokens)
    order, counts = dispatch(torch.from_numpy(ids).to(DEV), experts)
    assert np.array_equal(order.cpu().numpy().astype(np.int64), R.dispatch_order(ids))
    assert np.array_equal(counts.cpu().numpy().astype(np.int64), R.pair_counts(ids, experts))


def test_dispatch_severe_imbalance():
    # One expert with 4096 pairs, 199 with one pair each (reference test_grouped_buckets.py:146-189).
    ids = np.concatenate([np.zeros(4096, np.int64), np.arange(1, 200, dtype=np.int64)])[:, None]
    order, counts = dispatch(torch.from_numpy(ids).to(DEV), 200)
    assert np.array_equal(order.cpu().numpy().astype(np.int64), R.dispatch_order(ids))
    assert counts.cpu().numpy()[0] == 4096 and counts.cpu().numpy()[1:].tolist() == [1] * 199


def _run_layer(mixer, x_bits, batch, seq, logits_bits=None):
    x = from_bits(x_bits, DEV).reshape(batch, seq, -1)
    kw = {}
    if logits_bits is not None:
        kw["router_logits"] = from_bits(logits_bits, DEV).reshape(batch, seq, -1)
    with torch.no_grad():
        out = mixer(x, **kw)
    torch.cuda.synchronize()
    assert mixer.device_status() == 0
    return out


@pytest.mark.parametrize("name", LAYER_CASES)
def test_layer_with_reference_logits_matches_reference(name):
    arrays, meta = load_layer_case(name)
    mixer = build_mixer(meta, DEV)
    batch, seq = meta["shape"]
    out = _run_layer(mixer, arrays["x"], batch, seq, arrays["logits"])
    m = out.metrics
    k = meta["config"]["active_experts"]
    assert np.array_equal(bf16_bits(m["router_scores"]).reshape(-1, arrays["logits"].shape[1]),
                          arrays["router_scores"])
    assert np.array_equal(m["expert_ids"].cpu().numpy().reshape(-1, k), arrays["expert_ids"].astype(np.int64))
    assert np.array_equal(bf16_bits(m["routing_weights"]).reshape(-1, k), arrays["routing_weights"])
    assert np.array_equal(m["expert_utilization"].cpu().numpy().view(np.uint32),
                          arrays["expert_utilization"].view(np.uint32))
    for key, value in meta["scalars"].items():
        assert float(m[key]) == pytest.approx(value, rel=0, abs=0), key
    assert float(out.auxiliary_loss.float()) == pytest.approx(meta["aux_bf16"], rel=RTOL, abs=ATOL)
    assert_close_bf16(bf16_bits(out.update).reshape(arrays["update"].shape), arrays["update"])


@pytest.mark.parametrize("name", LAYER_CASES)
def test_layer_end_to_end_against_reference(name):
    """Own router GEMM: report routing agreement, update within tolerance."""

    arrays, meta = load_layer_case(name)
    mixer = build_mixer(meta, DEV)
    batch, seq = meta["shape"]
    out = _run_layer(mixer, arrays["x"], batch, seq)
    k = meta["config"]["active_experts"]
    ids = out.metrics["expert_ids"].cpu().numpy().reshape(-1, k)
    agree = float((ids == arrays["expert_ids"]).all(axis=1).mean())
    assert agree >= 0.95, f"routing agreement {agree:.4f}"
    # Against the oracle given the GPU's own routing: tolerance on every element.
    params = oracle_params(mixer)
    weights = bf16_bits(out.metrics["routing_weights"]).reshape(-1, k)
    routed, _, _ = R.grouped_experts(arrays["x"], ids, weights, params.gate, params.up, params.down,
                                     execution=meta["config"]["expert_execution"])
    want = routed
    if params.shared_gate is not None:
        shared = R.shared_swiglu(arrays["x"], params.shared_gate, params.shared_up, params.shared_down)
        want = R.f32_to_bf16_bits(bf16_bits_to_f32(routed) + bf16_bits_to_f32(shared))
    assert_close_bf16(bf16_bits(out.update).reshape(want.shape), want)


def _oracle_update_subset(params, x_bits, ids, weight_bits, tokens):
    """Oracle update rows for a subset of tokens given the layer's routing."""

    sub_ids = ids[tokens]
    sub_w = weight_bits[tokens]
    routed, _, _ = R.grouped_experts(x_bits[tokens], sub_ids, sub_w, params.gate, params.up, params.down)
    if params.shared_gate is None:
        return routed
    shared = R.shared_swiglu(x_bits[tokens], params.shared_gate, params.shared_up, params.shared_down)
    return R.f32_to_bf16_bits(bf16_bits_to_f32(routed) + bf16_bits_to_f32(shared))


FULL_CONFIGS = {
    "smoke": (dict(d_model=128, num_experts=200, expert_inter_dim=32, shared_inter_dim=128, active_experts=4), (2, 256)),
    "m10": (dict(d_model=256, num_experts=200, expert_inter_dim=64, shared_inter_dim=256, active_experts=8), (32, 512)),
    "m100": (dict(d_model=768, num_experts=200, expert_inter_dim=128, shared_inter_dim=768, active_experts=8), (64, 1024)),
}


@pytest.mark.parametrize("name", list(FULL_CONFIGS))
def test_full_size_layer_properties(name):
    cfg_kw, (batch, seq) = FULL_CONFIGS[name]
    config = MicroExpertsConfig(**cfg_kw)
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(DEV)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(batch, seq, config.d_model, generator=gen).to(torch.bfloat16)
    x_bits = bf16_bits(x).reshape(-1, config.d_model)
    out = _run_layer(mixer, x_bits, batch, seq)
    m = out.metrics
    E, k = config.num_experts, config.active_experts
    scores = bf16_bits(m["router_scores"]).reshape(-1, E)
    ids = m["expert_ids"].cpu().numpy().reshape(-1, k)
    # (1) selection is exactly the CPU top-k of the layer's own scores
    assert np.array_equal(topk_least(bf16_bits_to_f32(scores), k), ids)
    # (2) scores agree with the oracle router within one BF16 step of accumulation noise
    params = oracle_params(mixer)
    want_scores = R.router_scores(R.router_logits(x_bits, params.router_w, params.router_b))
    assert_close_bf16(scores, want_scores, rtol=1e-2, atol=1e-2)
    # (3) routing weights are the exact softmax of the selected scores
    sel = np.take_along_axis(scores, ids, axis=1)
    assert np.array_equal(bf16_bits(m["routing_weights"]).reshape(-1, k), R.routing_softmax(sel))
    # (4) dispatch permutation / counts / telemetry
    order, counts = dispatch(m["expert_ids"].reshape(-1, k), E)
    assert np.array_equal(order.cpu().numpy().astype(np.int64), R.dispatch_order(ids))
    ref_metrics = R.execution_metrics(ids, E)
    for key, value in ref_metrics.items():
        assert float(m[key]) == pytest.approx(value, rel=1e-7), key
    # (5) auxiliary loss from the layer's own scores and ids
    assert float(out.auxiliary_loss.float()) == pytest.approx(R.load_balance_loss(scores, ids), rel=RTOL, abs=ATOL)
    # (6) update rows on a token sample
    rng = np.random.default_rng(5)
    sample = np.sort(rng.choice(batch * seq, size=min(384, batch * seq), replace=False))
    weights = bf16_bits(m["routing_weights"]).reshape(-1, k)
    want = _oracle_update_subset(params, x_bits, ids, weights, sample)
    got = bf16_bits(out.update).reshape(-1, config.d_model)[sample]
    assert_close_bf16(got, want)
    # (7) every update row against the FP32 torch restatement on the device
    full = torch_layer_update(mixer, from_bits(x_bits, DEV), m["expert_ids"].reshape(-1, k),
                              m["routing_weights"].reshape(-1, k))
    # (the FP32 sums differ in order only: atol 1e-3 holds with room at these widths)
    assert_close_bf16(bf16_bits(out.update).reshape(-1, config.d_model), bf16_bits(full), atol=1e-3)


def test_layer_is_deterministic():
    cfg_kw, (batch, seq) = FULL_CONFIGS["m10"]
    config = MicroExpertsConfig(**cfg_kw)
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(DEV)
    x = torch.randn(batch, seq, config.d_model, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    x_bits = bf16_bits(x).reshape(-1, config.d_model)
    a = _run_layer(mixer, x_bits, batch, seq)
    b = _run_layer(mixer, x_bits, batch, seq)
    assert torch.equal(a.update, b.update)
    assert torch.equal(a.metrics["expert_ids"], b.metrics["expert_ids"])
    assert torch.equal(a.auxiliary_loss, b.auxiliary_loss)


def test_weights_repack_after_load_state_dict():
    cfg_kw, (batch, seq) = FULL_CONFIGS["smoke"]
    config = MicroExpertsConfig(**cfg_kw)
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(DEV)
    torch.manual_seed(1)
    other = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(DEV)
    x = torch.randn(batch, seq, config.d_model, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    x_bits = bf16_bits(x).reshape(-1, config.d_model)
    first = _run_layer(mixer, x_bits, batch, seq).update.clone()
    mixer.load_state_dict(other.state_dict())
    second = _run_layer(mixer, x_bits, batch, seq).update
    third = _run_layer(other, x_bits, batch, seq).update
    assert not torch.equal(first, second)
    assert torch.equal(second, third)
