"""Pin the CPU oracle against fixtures produced by the reference itself.

Runs on CPU.  Every later GPU parity test trusts the oracle only because these
checks pass: with the reference's own router logits injected, the oracle must
reproduce the reference's scores, expert ids (including tie order), routing
weights, dispatch permutation, counts, telemetry scalars and auxiliary loss
bit-exactly, and the layer update within the BF16 tolerance.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from oracle import mixer_ref as R
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits
from oracle.topk import topk_least
from tests.conftest import LAYER_CASES, load_layer_case
from tests.golden.topk_cases import TOPK_CASES, generate_scores
from tests.helpers import build_mixer, digest, oracle_params, resident_mask

RTOL, ATOL = 2e-2, 1e-2  # north_star BF16 tolerance


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.normal(0, 1, 100000).astype(np.float32),
        rng.normal(0, 1e-30, 1000).astype(np.float32),
        np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, 3.4e38, -3.4e38], dtype=np.float32),
    ])
    ours = f32_to_bf16_bits(vals)
    theirs = torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    nan = np.isnan(vals)
    assert np.array_equal(ours[~nan], theirs[~nan])
    assert np.all(np.isnan(bf16_bits_to_f32(ours[nan])))  # NaN payloads may differ


def test_softplus_table_matches_torch_on_every_bf16_input():
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    torch_out = torch.nn.functional.softplus(bits).view(torch.int16).numpy().view(np.uint16)
    ours = R.softplus_lut()
    finite = np.isfinite(bf16_bits_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16)))
    assert np.array_equal(ours[finite], torch_out[finite])
    nan_in = ~finite & np.isnan(bf16_bits_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16)))
    assert np.all(np.isnan(bf16_bits_to_f32(ours[nan_in])))


@pytest.mark.parametrize("case", TOPK_CASES, ids=[c["name"] for c in TOPK_CASES])
def test_oracle_topk_tie_order_matches_reference(case, golden_topk):
    scores, mask = generate_scores(case)
    digest_hex = hashlib.sha256(scores.tobytes()).hexdigest()
    assert digest_hex == bytes(golden_topk[f"{case['name']}__sha256"]).decode(), "generator drifted"
    eligible = bf16_bits_to_f32(scores).copy()
    if mask is not None:
        eligible[:, ~mask] = np.inf
    for k in case["ks"]:
        got = topk_least(eligible, k)
        assert np.array_equal(got, golden_topk[f"{case['name']}__k{k}"].astype(np.int64)), k


@pytest.mark.parametrize("name", LAYER_CASES)
def test_seeded_module_reproduces_reference_weights(name):
    arrays, meta = load_layer_case(name)
    mixer = build_mixer(meta)
    sd = mixer.state_dict()
    assert set(sd) == set(meta["digests"]), "state_dict keys differ from the reference"
    for key, expected in meta["digests"].items():
        assert digest(sd[key]) == expected, key


@pytest.mark.parametrize("name", LAYER_CASES)
def test_oracle_layer_matches_reference(name):
    arrays, meta = load_layer_case(name)
    cfg = meta["config"]
    mixer = build_mixer(meta)
    params = oracle_params(mixer)
    out = R.mixer_forward(
        params, arrays["x"], cfg["active_experts"], resident_mask=resident_mask(meta),
        transform=cfg["router_score_transform"], logit_bits=arrays["logits"],
        execution=cfg["expert_execution"],
    )
    assert np.array_equal(out["router_scores"], arrays["router_scores"])
    assert np.array_equal(out["expert_ids"], arrays["expert_ids"].astype(np.int64))
    assert np.array_equal(out["routing_weights"], arrays["routing_weights"])
    assert np.array_equal(out["order"], arrays["order"].astype(np.int64))
    assert np.array_equal(out["counts"], arrays["counts"].astype(np.int64))
    assert np.array_equal(out["expert_utilization"].view(np.uint32),
                          arrays["expert_utilization"].view(np.uint32))
    for key, value in meta["scalars"].items():
        assert out[key] == pytest.approx(value, rel=0, abs=0), key
    assert out["auxiliary_loss"] == meta["aux_bf16"]
    assert R.isclose_bf16(out["update"], arrays["update"], RTOL, ATOL)
    # The oracle reduces as the reference's index_add calls do (FP32 per call,
    # one BF16 rounding): it differs only by GEMM accumulation order.
    assert float((out["update"] == arrays["update"]).mean()) >= 0.99
    # Without injection, the oracle's own router GEMM differs only by accumulation order.
    own = R.router_logits(arrays["x"], params.router_w, params.router_b)
    diff = np.abs(bf16_bits_to_f32(own) - bf16_bits_to_f32(arrays["logits"]))
    assert float(diff.max()) <= 2.0 ** -6
