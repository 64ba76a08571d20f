"""GPU: spx_surprise_calibration against the reference's own outputs
(tests/golden/calibration.npz) and the oracle at a full-size shape."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle.calibration import surprise_calibration
from spalmer_b200.telemetry import attach_surprise_telemetry, layer_calibration
from tests.conftest import GOLDEN
from tests.helpers import from_bits

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("name", ("smoke", "m10_slice", "bias_resident", "k2_routed_only"))
def test_calibration_matches_reference_fixture(name):
    g = np.load(GOLDEN / "calibration.npz")
    z = np.load(GOLDEN / f"layer_{name}.npz")
    B, S = json.loads(bytes(z["meta"]).decode())["shape"]
    E = z["router_scores"].shape[-1]
    k = z["expert_ids"].shape[-1]
    metrics = {
        "router_scores": from_bits(z["router_scores"], DEV).reshape(B, S, E),
        "expert_ids": torch.from_numpy(z["expert_ids"].astype(np.int64)).to(DEV).reshape(B, S, k),
        "routing_weights": from_bits(z["routing_weights"], DEV).reshape(B, S, k),
    }
    nll = torch.from_numpy(g[f"{name}_nll"]).to(DEV)
    valid = torch.from_numpy(g[f"{name}_valid"]).to(DEV)
    enriched, total = attach_surprise_telemetry([metrics], nll, valid)
    np.testing.assert_allclose(float(total), g[f"{name}_calibration"][0], rtol=1e-5)
    np.testing.assert_allclose(enriched[0]["expert_attributed_nll"].cpu().numpy(), g[f"{name}_attributed_nll"],
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(enriched[0]["potentiation_utilization"].cpu().numpy(), g[f"{name}_utilization"],
                               rtol=1e-5, atol=1e-7)


def test_calibration_full_size_against_oracle_and_deterministic():
    B, S, E, k = 64, 1024, 200, 8
    rng = np.random.default_rng(7)
    scores = rng.random((B, S, E), dtype=np.float32) * 2
    scores_t = torch.from_numpy(scores).to(torch.bfloat16)
    ids = np.argsort(rng.random((B, S, E)), axis=-1)[..., :k].astype(np.int64)
    w = torch.softmax(torch.from_numpy(rng.standard_normal((B, S, k)).astype(np.float32)), -1).to(torch.bfloat16)
    nll = torch.from_numpy(rng.random((B, S - 1), dtype=np.float32) * 6)
    valid = torch.from_numpy(rng.random((B, S - 1)) > 0.05)
    args = (scores_t.to(DEV), torch.from_numpy(ids).to(DEV), w.to(DEV), nll.to(DEV), valid.to(DEV))
    cal, att, util = layer_calibration(*args)
    cal2, att2, util2 = layer_calibration(*args)
    assert torch.equal(att, att2) and torch.equal(util, util2) and torch.equal(cal, cal2)
    bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    want = surprise_calibration(bits(scores_t), ids, bits(w), nll.numpy(), valid.numpy())
    np.testing.assert_allclose(float(cal), want[0], rtol=1e-5)
    np.testing.assert_allclose(att.cpu().numpy(), want[1], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(util.cpu().numpy(), want[2], rtol=1e-4, atol=1e-8)
