"""Fit the router-bias scale alpha of the skewed expert-parallel config.

The bias b_e = alpha * ln(rank_e) over a seeded permutation of expert ids
(`make_golden.zipf_bias`) makes expert popularity fall with rank.  alpha is
chosen by bisection so the realised slot popularity tracks Zipf(s = 1.1):
the least-squares slope of log(share) against log(rank) over ranks 2..100
equals -1.1 (rank 1 is excluded: with k distinct experts per token a single
expert's share saturates at 1/k).  Routing uses the configuration's seed-0
router weights and 4096 seeded N(0, 1) tokens; writes zipf_ep_skew.json.

    python tests/golden/fit_zipf.py
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
import sys  # noqa: E402

sys.path.insert(0, str(ROOT))

from tests.golden.make_golden import zipf_bias  # noqa: E402

CFG = dict(d_model=1024, num_experts=200, expert_inter_dim=256, active_experts=8, router_bias=True)
TARGET = -1.1


def realised_shares(logits_f32: np.ndarray, bias: np.ndarray, k: int) -> np.ndarray:
    scores = np.logaddexp(0.0, logits_f32 + bias)  # softplus
    idx = np.argpartition(scores, k, axis=1)[:, :k]
    counts = np.bincount(idx.reshape(-1), minlength=scores.shape[1]).astype(np.float64)
    return counts / counts.sum()


def slope(shares_by_rank: np.ndarray) -> float:
    r = np.arange(2, 101)
    s = np.maximum(shares_by_rank[r - 1], 1e-12)
    return float(np.polyfit(np.log(r), np.log(s), 1)[0])


def main() -> None:
    from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig

    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(MicroExpertsConfig(**CFG, shared_inter_dim=0))
    w = mixer.router.proj.weight.detach().to(torch.bfloat16).float().numpy()
    x = torch.randn(4096, CFG["d_model"], generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).float()
    logits = x.numpy() @ w.T
    E, k = CFG["num_experts"], CFG["active_experts"]
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(3)).numpy()
    rank_of = np.empty(E, dtype=np.int64)
    rank_of[perm] = np.arange(1, E + 1)

    def by_rank(alpha: float) -> np.ndarray:
        shares = realised_shares(logits, zipf_bias(E, alpha).numpy(), k)
        out = np.empty(E)
        out[rank_of - 1] = shares
        return out

    lo, hi = 0.0, 4.0
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        if slope(by_rank(mid)) > TARGET:  # not steep enough yet
            lo = mid
        else:
            hi = mid
    alpha = 0.5 * (lo + hi)
    shares = by_rank(alpha)
    out = {"alpha": alpha, "target_slope": TARGET, "fitted_slope": slope(shares),
           "max_over_mean_share": float(shares.max() * E), "shares_by_rank": [round(v, 6) for v in shares]}
    (Path(__file__).parent / "zipf_ep_skew.json").write_text(json.dumps(out, indent=1) + "\n")
    print(json.dumps({k: v for k, v in out.items() if k != "shares_by_rank"}))


if __name__ == "__main__":
    main()
