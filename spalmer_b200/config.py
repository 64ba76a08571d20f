"""Configuration of one micro-expert layer, field-compatible with the reference.

Mirrors ``MicroExpertsConfig`` (mESmaC/spalmer src/spalmer/experts/config.py:17-288):
same field names, defaults, resolved properties and validation errors, so a
reference config object (or ``dataclasses.asdict`` of one) can be used
unchanged.  The B200 layer also accepts a reference config instance directly.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Literal

EXPERT_WEIGHT_FORMATS = ("mxfp4", "nvfp4", "mxfp6", "mxfp8", "bfloat16", "float32")
EXPERT_ACTIVATION_FORMATS = ("mxfp8", "nvfp4", "bfloat16", "float32")


def _positive(name: str, value: int) -> None:
    if value <= 0:
        raise ValueError(f"{name} must be positive")


@dataclass(frozen=True, slots=True)
class MicroExpertsConfig:
    """Bank, shared-path and routing configuration (see the module docstring)."""

    d_model: int
    num_experts: int = 200
    expert_inter_dim: int | None = None
    shared_inter_dim: int | None = None
    active_experts: int = 2
    min_active_experts: int = 2
    max_active_experts: int = 20
    min_resident_experts: int | None = None
    max_resident_experts: int = 20
    expert_execution: Literal["grouped", "loop"] = "grouped"
    expert_weight_format: str = "bfloat16"
    expert_activation_format: str = "bfloat16"
    expert_master_dtype: Literal["bfloat16", "float32"] = "bfloat16"
    expert_qat_backend: Literal["auto", "native"] = "auto"
    expert_promotion_format: Literal["mxfp8", "bfloat16", "float32"] = "bfloat16"
    potentiation_budget: int = 0
    potentiation_ema_decay: float = 0.95
    potentiation_warmup_steps: int = 4
    potentiation_hold_steps: int = 8
    potentiation_hysteresis: float = 0.05
    router_score_transform: Literal["softplus", "identity"] = "softplus"
    router_bias: bool = False
    residency_increment: int = 2
    residency_min_gain: float = 0.02
    initializer_range: float = 0.02

    def __post_init__(self) -> None:
        for name in ("d_model", "num_experts", "min_active_experts", "max_active_experts"):
            _positive(name, getattr(self, name))
        if self.min_resident_experts is None:
            object.__setattr__(self, "min_resident_experts", max(2, self.active_experts))
        _positive("min_resident_experts", self.min_resident_experts)
        _positive("max_resident_experts", self.max_resident_experts)
        if self.expert_inter_dim is not None and self.expert_inter_dim <= 0:
            raise ValueError("expert_inter_dim must be positive when provided")
        if self.shared_inter_dim is not None and self.shared_inter_dim < 0:
            raise ValueError("shared_inter_dim must be non-negative when provided")
        if self.expert_execution not in {"grouped", "loop"}:
            raise ValueError("expert_execution must be 'grouped' or 'loop'")
        if self.expert_weight_format not in EXPERT_WEIGHT_FORMATS:
            raise ValueError(f"expert_weight_format must be one of {EXPERT_WEIGHT_FORMATS}")
        if self.expert_activation_format not in EXPERT_ACTIVATION_FORMATS:
            raise ValueError(f"expert_activation_format must be one of {EXPERT_ACTIVATION_FORMATS}")
        if self.expert_master_dtype not in {"bfloat16", "float32"}:
            raise ValueError("expert_master_dtype must be 'bfloat16' or 'float32'")
        if self.expert_qat_backend not in {"auto", "native"}:
            raise ValueError("expert_qat_backend must be 'auto' or 'native'")
        if self.expert_promotion_format not in {"mxfp8", "bfloat16", "float32"}:
            raise ValueError("expert_promotion_format must be 'mxfp8', 'bfloat16', or 'float32'")
        fmt = self.expert_weight_format
        if fmt in {"bfloat16", "float32"}:
            if self.expert_activation_format != fmt:
                raise ValueError(f"{fmt.upper()} expert weights require matching activations")
            if self.expert_master_dtype != fmt:
                raise ValueError(f"{fmt.upper()} expert execution requires matching master parameters")
            if self.potentiation_budget:
                raise ValueError(
                    f"{fmt.upper()} expert execution has no higher promotion tier; "
                    "potentiation_budget must be zero"
                )
            if self.expert_promotion_format != fmt:
                raise ValueError(f"{fmt.upper()} expert execution requires matching promotion format")
        else:
            allowed = {"mxfp8", "nvfp4"} if fmt == "nvfp4" else {"mxfp8"}
            if self.expert_activation_format not in allowed:
                expected = "NVFP4 or MXFP8" if fmt == "nvfp4" else "MXFP8"
                raise ValueError(f"{fmt.upper()} expert weights require {expected} activations")
            if self.expert_master_dtype != "bfloat16":
                raise ValueError("low-precision expert training requires one BF16 master parameter payload")
            if self.expert_promotion_format == "float32":
                raise ValueError("low-precision experts do not expose an FP32 promotion lane")
        if not 0 <= self.potentiation_budget <= self.num_experts:
            raise ValueError(
                "potentiation_budget must be between zero and num_experts; "
                f"got {self.potentiation_budget}"
            )
        if not 0 <= self.potentiation_ema_decay < 1:
            raise ValueError("potentiation_ema_decay must be in [0, 1)")
        _positive("potentiation_warmup_steps", self.potentiation_warmup_steps)
        _positive("potentiation_hold_steps", self.potentiation_hold_steps)
        if self.potentiation_hysteresis < 0:
            raise ValueError("potentiation_hysteresis must be non-negative")
        if self.router_score_transform not in {"softplus", "identity"}:
            raise ValueError("router_score_transform must be 'softplus' or 'identity'")
        if self.initializer_range <= 0:
            raise ValueError("initializer_range must be positive")
        _positive("residency_increment", self.residency_increment)
        if not math.isfinite(self.residency_min_gain):
            raise ValueError("residency_min_gain must be finite")
        if self.min_active_experts > self.max_active_experts:
            raise ValueError(
                f"min_active_experts ({self.min_active_experts}) cannot exceed "
                f"max_active_experts ({self.max_active_experts})"
            )
        if self.num_experts < self.min_active_experts:
            raise ValueError(
                f"num_experts ({self.num_experts}) cannot be below the minimum "
                f"active expert count ({self.min_active_experts})"
            )
        effective_max = min(self.max_active_experts, self.num_experts)
        if not self.min_active_experts <= self.active_experts <= effective_max:
            raise ValueError(
                f"active_experts must be in [{self.min_active_experts}, "
                f"{effective_max}]; got {self.active_experts}"
            )
        if self.min_resident_experts < self.active_experts:
            raise ValueError(
                f"min_resident_experts ({self.min_resident_experts}) cannot be below "
                f"active_experts ({self.active_experts}): every token needs k residents"
            )
        if self.min_resident_experts > self.num_experts:
            raise ValueError(
                f"min_resident_experts ({self.min_resident_experts}) cannot exceed "
                f"num_experts ({self.num_experts})"
            )
        if self.min_resident_experts > self.resident_cap:
            raise ValueError(
                f"min_resident_experts ({self.min_resident_experts}) cannot exceed the "
                f"resident cap ({self.resident_cap})"
            )

    @property
    def resolved_inter_dim(self) -> int:
        return self.expert_inter_dim if self.expert_inter_dim is not None else max(1, self.d_model // 2)

    @property
    def resolved_shared_inter_dim(self) -> int:
        return self.shared_inter_dim if self.shared_inter_dim is not None else 2 * self.d_model

    @property
    def resident_cap(self) -> int:
        return min(self.max_resident_experts, self.num_experts)

    @property
    def expert_parameters_per_layer(self) -> int:
        return 3 * self.d_model * self.resolved_inter_dim

    @property
    def shared_parameters_per_layer(self) -> int:
        return 3 * self.d_model * self.resolved_shared_inter_dim

    @property
    def expert_pool_parameters_per_layer(self) -> int:
        return self.num_experts * self.expert_parameters_per_layer


def coerce_config(config) -> MicroExpertsConfig:
    """Accept this config, a reference ``MicroExpertsConfig`` or a mapping of its fields."""

    if isinstance(config, MicroExpertsConfig):
        return config
    if isinstance(config, dict):
        return MicroExpertsConfig(**config)
    fields = MicroExpertsConfig.__dataclass_fields__
    try:
        values = {name: getattr(config, name) for name in fields}
    except AttributeError as error:
        raise TypeError(f"not a MicroExpertsConfig: {type(config).__name__}") from error
    return MicroExpertsConfig(**values)
