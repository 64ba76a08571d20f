"""Golden vectors for the router's calibration loss term and the NLL
attribution (mESmaC/spalmer src/spalmer/modeling.py:1468-1534), produced by
running the reference functions themselves on the committed layer fixtures.

    python tests/golden/make_calibration.py /path/to/reference/src

For each layer case the inputs are the fixture's router_scores, expert_ids and
routing_weights ([B, S, .]), a seeded token NLL [B, S-1] (float32, uniform in
[0, 8)) and a seeded validity mask [B, S-1] (about 10% invalid); the outputs
are the per-layer calibration loss, expert_attributed_nll and
potentiation_utilization.  Writes calibration.npz next to this file.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
CASES = ("smoke", "m10_slice", "bias_resident", "k2_routed_only")


def _from_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.bfloat16)


def main() -> None:
    if len(sys.argv) > 1:
        sys.path.insert(0, sys.argv[1])
    from spalmer.modeling import _attach_surprise_telemetry

    out = {}
    for i, name in enumerate(CASES):
        z = np.load(HERE / f"layer_{name}.npz")
        meta = json.loads(bytes(z["meta"]).decode())
        B, S = meta["shape"]
        E = z["router_scores"].shape[-1]
        k = z["expert_ids"].shape[-1]
        scores = _from_bits(z["router_scores"]).reshape(B, S, E)
        ids = torch.from_numpy(z["expert_ids"].astype(np.int64)).reshape(B, S, k)
        weights = _from_bits(z["routing_weights"]).reshape(B, S, k)
        g = torch.Generator().manual_seed(100 + i)
        nll = torch.rand(B, S - 1, generator=g) * 8.0
        valid = torch.rand(B, S - 1, generator=g) >= 0.1
        metrics = {"router_scores": scores, "expert_ids": ids, "routing_weights": weights}
        enriched, total = _attach_surprise_telemetry([metrics], nll, valid)
        out[f"{name}_nll"] = nll.numpy()
        out[f"{name}_valid"] = valid.numpy()
        out[f"{name}_calibration"] = np.array([float(total)], dtype=np.float32)
        out[f"{name}_attributed_nll"] = enriched[0]["expert_attributed_nll"].numpy()
        out[f"{name}_utilization"] = enriched[0]["potentiation_utilization"].numpy()
    np.savez_compressed(HERE / "calibration.npz", **out)
    print("wrote calibration.npz", sorted(out))


if __name__ == "__main__":
    main()
