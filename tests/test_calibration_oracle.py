"""CPU: the calibration / attribution restatement against the reference's own
outputs (tests/golden/calibration.npz, made by tests/golden/make_calibration.py)."""

from __future__ import annotations

import json

import numpy as np
import pytest

from oracle.calibration import surprise_calibration
from tests.conftest import GOLDEN

CASES = ("smoke", "m10_slice", "bias_resident", "k2_routed_only")


@pytest.mark.parametrize("name", CASES)
def test_calibration_matches_reference(name):
    g = np.load(GOLDEN / "calibration.npz")
    z = np.load(GOLDEN / f"layer_{name}.npz")
    B, S = json.loads(bytes(z["meta"]).decode())["shape"]
    E = z["router_scores"].shape[-1]
    k = z["expert_ids"].shape[-1]
    cal, att, util = surprise_calibration(z["router_scores"].reshape(B, S, E), z["expert_ids"].reshape(B, S, k),
                                          z["routing_weights"].reshape(B, S, k), g[f"{name}_nll"], g[f"{name}_valid"])
    np.testing.assert_allclose(cal, g[f"{name}_calibration"][0], rtol=1e-6)
    np.testing.assert_allclose(att, g[f"{name}_attributed_nll"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(util, g[f"{name}_utilization"], rtol=1e-5, atol=1e-7)
