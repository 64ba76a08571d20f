"""The paged expert cache's host policy against traces of the reference itself
(tests/golden/paging_traces.json, made by tests/golden/make_paging.py from
mESmaC/spalmer experts/bank.py:241-365, 781-899): page plans, cached ids,
least-recently-used order and the four offload counters, call by call."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from spalmer_b200.offload import ExpertCachePolicy, page_plan, power_of_two_count_buckets

TRACES = json.loads((Path(__file__).parent / "golden" / "paging_traces.json").read_text())


@pytest.mark.parametrize("name", sorted(TRACES))
def test_policy_replays_reference_trace(name):
    case = TRACES[name]
    spec = case["spec"]
    E, cap = spec["num_experts"], spec["capacity"]
    policy = ExpertCachePolicy(E, cap, case["bytes_per_row"])
    if spec["warm"]:
        plan = policy.plan_rows(tuple(spec["warm"]))
        policy.commit(plan)
    assert list(policy.cached_ids) == case["warm"]["cached_ids"]
    assert policy.lru == case["warm"]["lru"]
    assert policy.counters == case["warm"]["counters"]
    for call in case["calls"]:
        counts = np.bincount(np.asarray(call["expert_index"]), minlength=E)
        pages = page_plan(counts, cap, loop=spec["execution"] == "loop")
        assert [list(p) for p in pages] == call["pages"]
        for page in pages:
            plan, lru = policy.plan_page(page)
            policy.commit(plan, lru)
            # every page's experts are resident, each in its own slot
            assert set(page) <= set(policy.cached_ids)
            slots = [policy.slots[e] for e in policy.cached_ids]
            assert len(set(slots)) == len(slots) and all(0 <= s < cap for s in slots)
        assert list(policy.cached_ids) == call["cached_ids"]
        assert policy.lru == call["lru"]
        assert policy.counters == call["counters"]


def test_retained_experts_keep_their_slots():
    policy = ExpertCachePolicy(10, 3, 8)
    policy.commit(policy.plan_rows((1, 4, 7)))
    before = dict(policy.slots)
    plan = policy.plan_rows((2, 4, 7))
    assert plan.incoming == ((2, before[1]),) and plan.evicted == (1,)
    policy.commit(plan)
    assert policy.slots[4] == before[4] and policy.slots[7] == before[7]
    assert policy.plan_rows((2, 4, 7)) is None  # no change, no stage operation
    forced = policy.plan_rows((2, 4, 7), force=True)
    assert [e for e, _ in forced.incoming] == [2, 4, 7] and forced.evicted == ()


def test_policy_validation_matches_reference_errors():
    policy = ExpertCachePolicy(6, 2, 8)
    with pytest.raises(ValueError, match="at least one"):
        policy.plan_rows(())
    with pytest.raises(ValueError, match="exceed cache capacity"):
        policy.plan_rows((0, 1, 2))
    with pytest.raises(ValueError, match="unique and sorted"):
        policy.plan_rows((3, 1))
    with pytest.raises(ValueError, match="must lie in"):
        policy.plan_rows((0, 6))
    with pytest.raises(ValueError, match="exceed cache capacity"):
        policy.plan_page((0, 1, 2))
    with pytest.raises(ValueError, match="capacity must lie"):
        ExpertCachePolicy(6, 7, 8)


def test_count_buckets():
    assert power_of_two_count_buckets([1, 3, 4, 5, 2, 8]) == ((1, (0,)), (2, (4,)), (4, (1, 2)), (8, (3, 5)))
    with pytest.raises(ValueError):
        power_of_two_count_buckets([1, 0])
    # loop pages are sorted selected ids; grouped pages follow the buckets
    counts = np.array([0, 5, 1, 0, 2, 9, 1])
    assert page_plan(counts, 2, loop=True) == [(1, 2), (4, 5), (6,)]
    assert page_plan(counts, 2) == [(2, 6), (4,), (1,), (5,)]


def test_enable_offload_argument_checks_on_host():
    import torch

    from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig
    from spalmer_b200.offload import enable_expert_offload

    config = MicroExpertsConfig(d_model=64, num_experts=8, expert_inter_dim=32, shared_inter_dim=64,
                                active_experts=2)
    mixer = B200MicroExpertChannelMixer(config)
    with pytest.raises(RuntimeError, match="inference-only"):
        enable_expert_offload(mixer.train(), "cuda:0", cache_size=4)
    mixer.eval()
    with pytest.raises(ValueError, match="CUDA"):
        enable_expert_offload(mixer, "cpu", cache_size=4)
    with pytest.raises(ValueError, match="cache_size must lie"):
        enable_expert_offload(mixer, "cuda:0", cache_size=9)
    with pytest.raises(ValueError, match="at least active_experts"):
        enable_expert_offload(mixer, "cuda:0", cache_size=4, resident_ids=(1,), paging=False)
    assert not mixer.experts.expert_offload_enabled
    assert getattr(mixer, "_expert_offload_manager", None) is None
    with pytest.raises(RuntimeError, match="inference-only"):
        mixer.train().experts._prepare_expert_offload(torch.device("cuda", 0), capacity=2, non_blocking=True,
                                                      pin_memory=False, paging=True)
