"""Paged expert offload on the GPU: the layer with its expert bank on the CPU
behind a bounded device cache (spx_layer_paged_begin / _experts / _finish,
spalmer_b200.offload) must give the unpaged layer's outputs bit for bit at
every cache size, in both precision lanes and batch classes, while its cache
follows the reference's paging policy (replayed on the host from the routed
expert counts).  Mirrors mESmaC/spalmer tests/experts/test_paged_offload.py."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig
from spalmer_b200.offload import (
    ExpertCachePolicy,
    disable_expert_offload,
    enable_expert_offload,
    expert_offload_telemetry,
    page_plan,
)
from tests.helpers import mxfp8_config, mxfp8_experts, set_mxfp8_lanes

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

M10 = dict(d_model=256, num_experts=64, expert_inter_dim=64, shared_inter_dim=256, active_experts=8)
KEYS = ("expert_ids", "routing_weights", "router_scores", "expert_utilization", "expert_group_count",
        "expert_group_max_load", "expert_group_real_pairs", "expert_group_padded_pairs", "expert_quantization_error")


def make_pair(config, seed=0, lanes=None):
    mixers = []
    for _ in range(2):
        torch.manual_seed(seed)
        m = B200MicroExpertChannelMixer(config).to(torch.bfloat16).to(DEV).eval()
        if lanes is not None:
            set_mxfp8_lanes(m, lanes)
        mixers.append(m)
    return mixers


def hidden(shape, d, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, d, generator=g).to(torch.bfloat16).to(DEV)


def assert_same(got, want):
    assert torch.equal(got.update, want.update)
    assert torch.equal(got.auxiliary_loss, want.auxiliary_loss)
    for key in KEYS:
        assert torch.equal(got.metrics[key], want.metrics[key]), key


def replay(policy: ExpertCachePolicy, ids: torch.Tensor, E: int, capacity: int, loop=False):
    counts = np.bincount(ids.reshape(-1).cpu().numpy(), minlength=E)
    for page in page_plan(counts, capacity, loop=loop):
        policy.commit(*policy.plan_page(page))


@pytest.mark.parametrize("capacity", [64, 20, 7, 1])
@pytest.mark.parametrize("shape", [(2, 512), (1, 64)], ids=["prefill", "decode_class"])
def test_paged_matches_unpaged(capacity, shape):
    config = MicroExpertsConfig(**M10)
    ref_mixer, paged = make_pair(config)
    telemetry = enable_expert_offload(paged, DEV, cache_size=capacity)
    assert telemetry.paging and telemetry.masters_on_cpu and telemetry.masters_pinned
    assert paged.experts.gate_proj.device.type == "cpu" and paged.router.proj.weight.device == DEV
    policy = ExpertCachePolicy(config.num_experts, capacity, paged.experts.parameters_per_expert * 2)
    for step in range(3):
        x = hidden(shape, config.d_model, seed=1 + step % 2)
        with torch.no_grad():
            want = ref_mixer(x)
        got = paged(x)  # grad mode on: offload is inference-only and records no graph
        assert_same(got, want)
        assert got.metrics["expert_paging"] is True
        replay(policy, want.metrics["expert_ids"], config.num_experts, capacity)
        assert paged.experts.cached_expert_ids == policy.cached_ids
        assert paged.experts.expert_offload_counters == tuple(policy.counters)
    assert paged.device_status() == 0
    assert len(paged.experts.cached_expert_ids) <= capacity


def test_paged_mxfp8_lane_matches_unpaged():
    config = mxfp8_config(**M10)
    lanes = mxfp8_experts(config.num_experts, 0.25)
    ref_mixer, paged = make_pair(config, lanes=lanes)
    enable_expert_offload(paged, DEV, cache_size=24)
    x = hidden((2, 512), config.d_model)
    with torch.no_grad():
        want = ref_mixer(x)
        got = paged(x)
    assert_same(got, want)
    assert paged.device_status() == 0


def test_decode_steps_hit_the_cache():
    config = MicroExpertsConfig(**M10)
    ref_mixer, paged = make_pair(config)
    enable_expert_offload(paged, DEV, cache_size=16, resident_ids=(0, 1, 2))
    assert paged.experts.cached_expert_ids == (0, 1, 2)
    x = hidden((1, 1), config.d_model)
    with torch.no_grad():
        first = paged(x)
        rows = paged.experts.expert_offload_counters[1]
        for _ in range(3):
            again = paged(x)
            assert_same(again, first)
        assert paged.experts.expert_offload_counters[1] == rows  # hits: nothing transferred
        assert_same(first, ref_mixer(x))


def test_masters_reloaded_refresh_the_cache():
    config = MicroExpertsConfig(**M10)
    ref_mixer, paged = make_pair(config)
    enable_expert_offload(paged, DEV, cache_size=32)
    x = hidden((2, 512), config.d_model)
    with torch.no_grad():
        paged(x)
        torch.manual_seed(5)
        other = B200MicroExpertChannelMixer(config).to(torch.bfloat16)
        state = other.state_dict()
        ref_mixer.load_state_dict(state)
        paged.load_state_dict(state)
        assert paged.experts.gate_proj.device.type == "cpu"
        assert_same(paged(x), ref_mixer(x))


def test_resident_mode_restricts_routing():
    config = MicroExpertsConfig(**M10)
    ref_mixer, paged = make_pair(config)
    residents = tuple(range(0, 64, 4))  # within the default resident cap
    telemetry = enable_expert_offload(paged, DEV, cache_size=len(residents), resident_ids=residents,
                                      paging=False)
    assert telemetry.mode == "resident" and telemetry.resident_expert_ids == residents
    ref_mixer.residency.set(residents)
    x = hidden((2, 512), config.d_model)
    with torch.no_grad():
        got, want = paged(x), ref_mixer(x)
    assert_same(got, want)
    assert set(got.metrics["expert_ids"].unique().tolist()) <= set(residents)
    assert got.metrics["expert_paging"] is False


def test_enable_disable_and_telemetry():
    config = MicroExpertsConfig(**M10)
    ref_mixer, paged = make_pair(config)
    container = torch.nn.Sequential(paged).eval()
    telemetry = enable_expert_offload(container, DEV, cache_size=8, resident_ids=(3, 5))
    assert telemetry.cached_expert_ids_by_layer == ((3, 5),)
    assert telemetry.occupancy == 0.25 and telemetry.caches_on_target
    assert telemetry.transferred_expert_rows == 2 and telemetry.stage_operations == 1
    with pytest.raises(RuntimeError, match="already enabled"):
        enable_expert_offload(container, DEV, cache_size=8)
    x = hidden((1, 64), config.d_model)
    with torch.no_grad():
        container(x)
    after = expert_offload_telemetry(container)
    assert after.stage_operations > telemetry.stage_operations
    disable_expert_offload(container, device=DEV)
    assert expert_offload_telemetry(container) is None
    assert paged.experts.gate_proj.device == DEV and not paged.experts.expert_offload_enabled
    with torch.no_grad():
        assert_same(paged(x), ref_mixer(x))


def test_stage_expert_slots_copies_whole_experts_from_host():
    from spalmer_b200 import _lib

    lib = _lib.load()
    E, C = 12, 5
    g = torch.Generator().manual_seed(3)
    host = [torch.randint(0, 255, (E, n), generator=g, dtype=torch.uint8).pin_memory() for n in (4096, 1040)]
    dev = [torch.zeros(C, t.shape[1], dtype=torch.uint8, device=DEV) for t in host]
    pairs = [(7, 2), (0, 4), (11, 0), (3, 9), (-1, 1)]  # the last two are out of range: skipped
    pairs_dev = torch.tensor(pairs, dtype=torch.int32, device=DEV)
    src = (_lib.ctypes.c_void_p * 2)(*(t.data_ptr() for t in host))
    dst = (_lib.ctypes.c_void_p * 2)(*(t.data_ptr() for t in dev))
    nbytes = (_lib.ctypes.c_int64 * 2)(*(t.shape[1] for t in host))
    stream = torch.cuda.current_stream(DEV).cuda_stream
    assert lib.spx_stage_expert_slots(src, dst, nbytes, 2, pairs_dev.data_ptr(), len(pairs), E, C, 4, stream) == 0
    torch.cuda.synchronize()
    for h, d in zip(host, dev):
        for e, s in pairs[:3]:
            assert torch.equal(d[s].cpu(), h[e])
        assert not d[1].any() and not d[3].any()
    # pageable host memory cannot be read by the device: refused before any launch
    pageable = torch.zeros(E, 4096, dtype=torch.uint8)
    src_bad = (_lib.ctypes.c_void_p * 1)(pageable.data_ptr())
    nb = (_lib.ctypes.c_int64 * 1)(4096)
    dst1 = (_lib.ctypes.c_void_p * 1)(dev[0].data_ptr())
    assert lib.spx_stage_expert_slots(src_bad, dst1, nb, 1, pairs_dev.data_ptr(), 3, E, C, 0, stream) == -1


def test_paged_nvfp4_lane_matches_unpaged():
    config = MicroExpertsConfig(**M10, expert_weight_format="nvfp4", expert_activation_format="nvfp4",
                                expert_promotion_format="bfloat16")
    lanes = mxfp8_experts(config.num_experts, 0.5)
    ref_mixer, paged = make_pair(config, lanes=lanes)
    enable_expert_offload(paged, DEV, cache_size=20)
    x = hidden((2, 512), config.d_model)
    with torch.no_grad():
        want = ref_mixer(x)
        got = paged(x)
    assert_same(got, want)
    assert paged.device_status() == 0
