"""Precision-provider hook for the reference's capability discovery.

The reference imports ``spalmer.experts.native.native_provider_capabilities``
(precision.py:396-430) and accepts claims with the fields of
``ExpertPrecisionCapability`` (precision.py:68-107).  This module returns the
claim of the B200 grouped kernels so a maintainer can forward that hook here.
The claim is verified by running one small layer on the device; the backward
pass does not exist yet, so ``backward_available`` is False and the reference
will not select this provider for training.
"""

from __future__ import annotations

from functools import lru_cache

import torch

PROVIDER_ID = "spx_sm100_grouped"


@lru_cache(maxsize=8)
def _smoke(device_index: int) -> tuple[bool, str]:
    from spalmer_b200.config import MicroExpertsConfig
    from spalmer_b200.experts import B200MicroExpertChannelMixer

    try:
        device = torch.device("cuda", device_index)
        major, minor = torch.cuda.get_device_capability(device)
        if (major, minor) != (10, 0):
            return False, f"sm_{major}{minor} is not sm_100"
        config = MicroExpertsConfig(d_model=128, num_experts=16, expert_inter_dim=32, active_experts=4,
                                    shared_inter_dim=128)
        with torch.no_grad():
            gen = torch.Generator().manual_seed(1204)
            mixer = B200MicroExpertChannelMixer(config).to(device=device, dtype=torch.bfloat16)
            x = torch.randn(1, 256, 128, generator=gen).to(device=device, dtype=torch.bfloat16)
            out = mixer(x)
            torch.cuda.synchronize(device)
            ok = bool(torch.isfinite(out.update.float()).all()) and mixer.device_status() == 0
        return ok, "libspx sm_100a grouped forward smoke " + ("passed" if ok else "failed")
    except Exception as error:  # noqa: BLE001 - report, never raise from discovery
        return False, f"libspx smoke failed: {error}"


def native_provider_capabilities(device: str | torch.device | None = None) -> list[dict[str, str | bool]]:
    resolved = torch.device(device if device is not None else ("cuda" if torch.cuda.is_available() else "cpu"))
    if resolved.type == "cuda" and resolved.index is None and torch.cuda.is_available():
        resolved = torch.device("cuda", torch.cuda.current_device())
    if resolved.type != "cuda" or not torch.cuda.is_available():
        available, detail = False, "CUDA is unavailable"
    else:
        available, detail = _smoke(resolved.index)
    return [
        {
            "provider_id": PROVIDER_ID,
            "weight_format": "bfloat16",
            "activation_format": "bfloat16",
            "forward_available": available,
            "backward_available": False,
            "grouped_available": available,
            "verified": available,
            "detail": detail,
        }
    ]
