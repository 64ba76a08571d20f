"""Pin the oracle's bank seam (``MicroExpertBank.execute_routing``,
experts/bank.py:593-646) against fixtures made by running the reference on
arbitrary routing pairs (``tests/golden/make_bank.py``): ragged pairs per
token, tokens without pairs, a token with 30 pairs, the grouped and the loop
executors, and a restricted resident set whose non-resident pairs the grouped
path does not execute.  CPU only."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import mixer_ref as R
from oracle.bf16 import bf16_bits_to_f32
from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig
from tests.conftest import GOLDEN
from tests.helpers import digest, oracle_params

RTOL, ATOL = 2e-2, 1e-2


def load_bank():
    z = np.load(GOLDEN / "bank_pairs.npz")
    arrays = {key: z[key] for key in z.files if key != "meta"}
    return arrays, json.loads(bytes(z["meta"]).decode())


def seeded_mixer(meta, execution="grouped", device=None):
    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(MicroExpertsConfig(**meta["config"], expert_execution=execution))
    mixer = mixer.to(torch.bfloat16).eval()
    return mixer if device is None else mixer.to(device)


def test_bank_weights_are_the_reference_bank():
    arrays, meta = load_bank()
    sd = seeded_mixer(meta).experts.state_dict()
    assert set(sd) == set(meta["digests"])
    for key, expected in meta["digests"].items():
        assert digest(sd[key]) == expected, key


@pytest.mark.parametrize("case", ["grouped", "loop", "resident"])
def test_oracle_execute_routing_matches_reference(case):
    arrays, meta = load_bank()
    params = oracle_params(seeded_mixer(meta))
    resident = arrays.get(f"{case}__resident_ids")
    got = R.execute_routing(arrays["x"], arrays[f"{case}__token_index"], arrays[f"{case}__expert_index"],
                            arrays[f"{case}__weights"], params.gate, params.up, params.down,
                            execution=meta["cases"][case]["execution"], resident_ids=resident)
    want = arrays[f"{case}__update"]
    a, b = bf16_bits_to_f32(got), bf16_bits_to_f32(want)
    assert np.all(np.abs(a - b) <= ATOL + RTOL * np.abs(b))
    # same reduction order as the reference: most elements agree bit for bit
    assert float((got == want).mean()) > 0.99
    if resident is not None:  # non-resident pairs dropped, rows of untouched tokens zero
        assert np.any(~np.isin(arrays[f"{case}__expert_index"], resident))
    assert not np.any(want[48:])
