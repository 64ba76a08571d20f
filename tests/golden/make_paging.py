"""Generate paging traces by running the reference's paged expert bank itself.

Run in the build container, where the reference source is importable::

    python tests/golden/make_paging.py /path/to/reference/src

The reference (mESmaC/spalmer) pages expert weights through a bounded cache
(``MicroExpertBank._prepare_expert_offload(..., paging=True)``,
``_stage_expert_rows``, ``_stage_execution_page``, experts/bank.py:195-365)
and executes unrestricted routing page by page (``_execute_paged_grouped`` /
``_execute_paged_loop``, bank.py:781-899).  Each case below builds a float32
bank on the CPU, optionally warms the cache, then calls ``execute_routing``
with a seeded sequence of routings.  Recorded per call: the expert index of
every pair (the input), the pages the bank staged (in order), and afterwards
the cached ids, the LRU order and the offload counters.  The B200 layer's
host-side cache policy must reproduce these traces from the per-expert pair
counts alone.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent

CASES = {
    # grouped execution, uneven loads over several power-of-two buckets,
    # more selected experts than cache rows
    "grouped_cap3": dict(num_experts=12, capacity=3, execution="grouped", warm=(0, 3), calls=8, tokens=9, k=2),
    "grouped_cap5": dict(num_experts=16, capacity=5, execution="grouped", warm=(), calls=8, tokens=24, k=3),
    # capacity one: every page a single expert
    "grouped_cap1": dict(num_experts=6, capacity=1, execution="grouped", warm=(), calls=5, tokens=4, k=2),
    # loop execution pages sorted selected ids directly
    "loop_cap4": dict(num_experts=12, capacity=4, execution="loop", warm=(1, 2), calls=8, tokens=7, k=2),
    # decode-like calls whose selections fit the cache (LRU hits)
    "decode_cap8": dict(num_experts=20, capacity=8, execution="grouped", warm=(), calls=10, tokens=1, k=4),
}


def make_case(name: str, spec: dict) -> dict:
    from spalmer.experts import MicroExpertBank, MicroExpertsConfig

    config = MicroExpertsConfig(
        d_model=8, num_experts=spec["num_experts"], expert_inter_dim=3, shared_inter_dim=4,
        active_experts=spec["k"], max_active_experts=spec["k"], max_resident_experts=spec["num_experts"],
        potentiation_budget=0, expert_execution=spec["execution"], expert_weight_format="float32",
        expert_activation_format="float32", expert_master_dtype="float32", expert_promotion_format="float32",
    )
    torch.manual_seed(0)
    bank = MicroExpertBank(config).eval()
    bank._prepare_expert_offload(torch.device("cpu"), capacity=spec["capacity"], non_blocking=False,
                                 pin_memory=False, paging=True)
    if spec["warm"]:
        bank._stage_expert_rows(tuple(spec["warm"]))
    warm = {"cached_ids": list(bank.cached_expert_ids), "lru": list(bank._cached_lru),
            "counters": list(bank.expert_offload_counters)}
    pages: list[list[int]] = []
    original = bank._stage_execution_page

    def recording(required_ids):
        pages.append(sorted(set(int(e) for e in required_ids)))
        return original(required_ids)

    bank._stage_execution_page = recording
    g = torch.Generator().manual_seed(sum(map(ord, name)))
    E, k, T = spec["num_experts"], spec["k"], spec["tokens"]
    # skewed popularity so that counts fall in several buckets
    popularity = torch.rand(E, generator=g) ** 3 + 0.02
    calls = []
    for _ in range(spec["calls"]):
        expert_ids = torch.stack([torch.multinomial(popularity, k, replacement=False, generator=g) for _ in range(T)])
        expert_index = expert_ids.reshape(-1)
        hidden = torch.randn(T, config.d_model, generator=g)
        token_index = torch.arange(T).repeat_interleave(k)
        weights = torch.full((T * k,), 1.0 / k)
        pages.clear()
        bank.execute_routing(hidden, token_index, expert_index, weights)
        calls.append({
            "expert_index": expert_index.tolist(),
            "pages": [list(p) for p in pages],
            "cached_ids": list(bank.cached_expert_ids),
            "lru": list(bank._cached_lru),
            "counters": list(bank.expert_offload_counters),
        })
    return {"spec": {**spec, "warm": list(spec["warm"])},
            "bytes_per_row": bank.parameters_per_expert * bank.gate_proj.element_size(),
            "warm": warm, "calls": calls}


def main() -> None:
    if len(sys.argv) > 1:
        sys.path.insert(0, sys.argv[1])
    out = {name: make_case(name, spec) for name, spec in CASES.items()}
    (HERE / "paging_traces.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", HERE / "paging_traces.json")


if __name__ == "__main__":
    main()
