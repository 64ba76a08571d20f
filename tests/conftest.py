"""pytest configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` runs on CPU (oracle pinning, host logic, ABI symbol checks);
`-m gpu` runs the parity tests against libspx on a B200.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"
LAYER_CASES = ("smoke", "m10_slice", "m100_slice", "k2_routed_only", "bias_resident", "tiny_identity",
               "smoke_loop", "m10_loop")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and libspx")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_layer_case(name: str) -> tuple[dict, dict]:
    z = np.load(GOLDEN / f"layer_{name}.npz")
    arrays = {key: z[key] for key in z.files if key != "meta"}
    meta = json.loads(bytes(z["meta"]).decode())
    return arrays, meta


@pytest.fixture(scope="session")
def golden_topk():
    z = np.load(GOLDEN / "topk_ties.npz")
    return {key: z[key] for key in z.files}
