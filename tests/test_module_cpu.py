"""Host-side behaviour of the drop-in module (no GPU needed)."""

from __future__ import annotations

import sys

import pytest
import torch

from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig, SurpriseRouter


def small_config(**kw):
    base = dict(d_model=64, num_experts=16, expert_inter_dim=16, active_experts=4)
    base.update(kw)
    return MicroExpertsConfig(**base)


def test_state_dict_keys_match_reference_layout():
    mixer = B200MicroExpertChannelMixer(small_config(shared_inter_dim=32))
    keys = set(mixer.state_dict())
    assert {
        "router.proj.weight", "experts.gate_proj", "experts.up_proj", "experts.down_proj",
        "shared.gate_projection.weight", "shared.up_projection.weight", "shared.down_projection.weight",
        "_owned_potentiation_controller.utilization_ema", "_owned_potentiation_controller.promoted_mask",
    } <= keys
    assert not any("resident" in k for k in keys)  # residency buffers are non-persistent
    assert mixer.experts.gate_proj.shape == (16, 64, 16)
    assert mixer.experts.down_proj.shape == (16, 16, 64)


def test_shared_router_validation_mirrors_reference():
    router = SurpriseRouter(small_config())
    with pytest.raises(ValueError, match="8"):
        B200MicroExpertChannelMixer(small_config(num_experts=8), router=router)
    layer1 = B200MicroExpertChannelMixer(small_config(), router=router)
    layer2 = B200MicroExpertChannelMixer(small_config(), router=router)
    assert layer1.router is layer2.router and layer1.experts is not layer2.experts


def test_forward_fails_loudly_off_gpu_with_and_without_autograd():
    mixer = B200MicroExpertChannelMixer(small_config()).to(torch.bfloat16)
    x = torch.randn(1, 4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        mixer(x)  # the training path has no CPU fallback either
    with pytest.raises(ValueError, match="router_logits"):
        mixer(x, router_logits=torch.zeros(1, 4, 16, dtype=torch.bfloat16))
    with torch.no_grad(), pytest.raises(RuntimeError, match="CUDA"):
        mixer(x)
    with torch.no_grad(), pytest.raises(ValueError):
        mixer(torch.randn(4, 64, dtype=torch.bfloat16))


def test_config_validation_matches_reference_messages():
    with pytest.raises(ValueError, match="potentiation_budget must be zero"):
        MicroExpertsConfig(d_model=8, potentiation_budget=2)
    with pytest.raises(ValueError, match="active_experts must be in"):
        MicroExpertsConfig(d_model=8, num_experts=4, active_experts=5)
    cfg = MicroExpertsConfig(d_model=8, num_experts=4, active_experts=3)
    assert cfg.min_resident_experts == 3
    assert cfg.resolved_inter_dim == 4 and cfg.resolved_shared_inter_dim == 16


def _reference_site() -> str | None:
    """The installed reference (baseline/_ref, oracle/install_ref.py) or
    $SPALMER_REFERENCE/src, when either exists."""

    import os
    from pathlib import Path

    site = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
    if (site / "spalmer").is_dir():
        return str(site)
    root = os.environ.get("SPALMER_REFERENCE")
    return str(Path(root) / "src") if root else None


def test_reference_config_objects_are_accepted():
    ref_src = _reference_site()
    if ref_src is None:
        pytest.skip("reference package not available")
    try:
        sys.path.insert(0, ref_src)
        from spalmer.experts import MicroExpertsConfig as RefConfig  # type: ignore
    except Exception:  # noqa: BLE001
        pytest.skip("reference package not importable here")
    finally:
        if sys.path and sys.path[0] == ref_src:
            sys.path.pop(0)
    ref = RefConfig(d_model=64, num_experts=16, expert_inter_dim=16, active_experts=4)
    mixer = B200MicroExpertChannelMixer(ref)
    assert mixer.config == small_config()
