"""The backward oracle (oracle/mixer_autograd.py) against the reference's own
gradients (tests/golden/backward_*.npz, written by make_backward.py)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import mixer_autograd as MA
from tests.helpers import build_mixer, digest, from_bits

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ("small", "large")


def load_backward_case(name: str):
    arrays = np.load(GOLDEN / f"backward_{name}.npz")
    meta = json.loads(bytes(arrays["meta"]).decode())
    return arrays, meta


def relnorm(got: torch.Tensor, want: torch.Tensor) -> float:
    want = want.float()
    return float((got.float() - want).norm() / want.norm().clamp_min(1e-30))


@pytest.mark.parametrize("name", CASES)
def test_backward_case_weights_regenerate_from_seed(name):
    _, meta = load_backward_case(name)
    sd = build_mixer(meta).state_dict()
    for key, expected in meta["digests"].items():
        assert digest(sd[key]) == expected, key


@pytest.mark.parametrize("name", CASES)
def test_oracle_gradients_match_reference(name):
    arrays, meta = load_backward_case(name)
    mixer = build_mixer(meta)
    sd = mixer.state_dict()
    params = {k: sd[k] for k in MA.PARAM_NAMES if k in sd}
    k = meta["config"]["active_experts"]
    grads = MA.gradients(params, from_bits(arrays["x"]), k, from_bits(arrays["d_update"]), meta["d_aux"])
    assert set(meta["grads"]) == set(params)
    for key in params:
        want = from_bits(arrays["grad__" + key])
        # Same ops, same order: the weight gradients agree to the last bit.
        assert torch.equal(grads[key], want), (key, relnorm(grads[key], want))
    # The input gradient sums the routed rows in a different order.
    assert relnorm(grads["x"], from_bits(arrays["grad_x"])) < 2e-2
