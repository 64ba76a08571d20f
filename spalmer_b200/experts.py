"""B200 drop-in for SPALMER's routed micro-expert channel mixer.

``B200MicroExpertChannelMixer`` (alias ``MicroExpertChannelMixer``) has the
constructor and ``forward`` contract of the reference module
(mESmaC/spalmer src/spalmer/experts/mixer.py:38-241) and the same
``state_dict`` keys and layouts, and a model built under the same
``torch.manual_seed`` holds bit-identical weights: the parameter-holding
submodules below create their parameters in the reference's order
(router ``nn.Linear`` + ``normal_``, bank ``randn`` x3, shared SwiGLU
``nn.Linear`` x3 + ``normal_``).

``forward`` runs one call of ``spx_layer_forward`` (libspx, sm_100a): router
GEMM, exact least-surprise top-k, dispatch, grouped expert SwiGLU, shared
SwiGLU fused with the combine, routing statistics and the load-balance loss,
with no host synchronisation.  There is no CPU or PyTorch fallback: inputs
must be BF16 CUDA tensors and the library must be built.  Under autograd the
same native forward runs inside an ``autograd.Function`` whose backward calls
``spx_layer_backward`` (BF16 experts).  With expert offload enabled
(``spalmer_b200.offload``) the expert bank stays on the CPU and the forward
pages the selected experts through a bounded device cache.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Mapping
from weakref import ref

import torch
from torch import Tensor, nn

from spalmer_b200 import _lib
from spalmer_b200.config import MicroExpertsConfig, coerce_config
from spalmer_b200.native import NativeExpertPrecisionError

try:  # the reference shell's output type, when the reference package is importable
    from spalmer.modeling import ChannelMixerOutput  # type: ignore
except Exception:  # noqa: BLE001 - optional integration

    @dataclass(slots=True)
    class ChannelMixerOutput:  # same fields as spalmer.modeling.ChannelMixerOutput (modeling.py:27-31)
        update: Tensor
        state: Any = None
        auxiliary_loss: Tensor | None = None
        metrics: Mapping[str, Any] = field(default_factory=dict)


# ---------------------------------------------------------------- parameter holders


class SurpriseRouter(nn.Module):
    """Router parameters and score transform (experts/router.py:19-56)."""

    def __init__(self, config) -> None:
        super().__init__()
        config = coerce_config(config)
        self.config = config
        self.num_experts = config.num_experts
        self.proj = nn.Linear(config.d_model, config.num_experts, bias=config.router_bias)
        nn.init.normal_(self.proj.weight, mean=0.0, std=config.initializer_range)
        if self.proj.bias is not None:
            nn.init.zeros_(self.proj.bias)

    @property
    def num_features(self) -> int:
        return self.config.d_model

    def forward(self, hidden_states: Tensor) -> Tensor:
        """Predicted surprise ``[..., experts]`` (experts/router.py:40-56):
        ``softplus(x @ W^T + b)`` in BF16, or the logits for the legacy
        identity transform, through ``spx_router_forward`` (the layer's
        tcgen05 router GEMM, then the BF16 softplus table).  Under autograd the
        gradients of x, W and b follow the reference's autograd steps."""

        if hidden_states.shape[-1] != self.config.d_model:
            raise ValueError(
                f"expected trailing dimension {self.config.d_model}, got {hidden_states.shape[-1]}"
            )
        params = [self.proj.weight] + ([self.proj.bias] if self.proj.bias is not None else [])
        if torch.is_grad_enabled() and (hidden_states.requires_grad or any(p.requires_grad for p in params)):
            return _RouterFunction.apply(self, hidden_states, *params)
        return self._scores(hidden_states, identity=False)

    def _scores(self, hidden_states: Tensor, *, identity: bool) -> Tensor:
        d, E = self.config.d_model, self.num_experts
        device = hidden_states.device
        if device.type != "cuda":
            raise RuntimeError(f"the B200 router executes CUDA tensors; hidden states are on {device}")
        w, b = self.proj.weight, self.proj.bias
        if hidden_states.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
            raise RuntimeError(
                f"the B200 router executes BF16; hidden states are {hidden_states.dtype}, weight {w.dtype}"
            )
        if w.device != device:
            raise RuntimeError(f"router weight is on {w.device}, hidden states on {device}")
        lead = hidden_states.shape[:-1]
        x = hidden_states.reshape(-1, d).contiguous()
        T = x.shape[0]
        out = torch.empty(T, E, dtype=torch.bfloat16, device=device)
        if T == 0:
            return out.reshape(*lead, E)
        lib = _lib.load()
        transform = 1 if identity or self.config.router_score_transform == "identity" else 0
        dims = _lib.LayerDims(tokens=T, d_model=d, num_experts=E, inter_dim=16, shared_dim=0, top_k=1,
                              score_transform=transform, execution_loop=0, mxfp8_lane=0)
        small = T <= SMALL_BATCH_TOKENS
        key = (device, small, w.data_ptr(), w._version)
        cache = self.__dict__.setdefault("_router_pack", {})
        packed = cache.get(small)
        if packed is None or packed[0] != key:
            sizes = _lib.PackedSizes()
            _lib.check(lib.spx_layer_sizes(dims, None, sizes), "spx_layer_sizes")
            pw = torch.empty(max(1, sizes.router_weight), dtype=torch.int16, device=device)
            wb = w.detach().contiguous()
            src = _lib.ReferenceWeights(router_weight=wb.data_ptr())
            _lib.check(lib.spx_pack_weights(dims, src, pw.data_ptr(), None, None, None, None,
                                            torch.cuda.current_stream(device).cuda_stream), "spx_pack_weights (router)")
            packed = (key, pw, wb)
            cache[small] = packed
        nbytes = _lib.ctypes.c_size_t()
        _lib.check(lib.spx_router_sizes(dims, nbytes), "spx_router_sizes")
        ws = self.__dict__.get("_router_ws")
        if ws is None or ws.device != device or ws.numel() < nbytes.value:
            ws = torch.zeros(nbytes.value, dtype=torch.uint8, device=device)
            self.__dict__["_router_ws"] = ws
        bias = None if b is None else b.detach().to(torch.bfloat16).contiguous()
        pwt = _lib.PackedWeights(router_weight=packed[1].data_ptr(), router_bias=_lib.ptr(bias),
                                 softplus_table=_lib.ptr(softplus_table(device)) if transform == 0 else None)
        _lib.check(lib.spx_router_forward(dims, pwt, x.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                          torch.cuda.current_stream(device).cuda_stream), "spx_router_forward")
        return out.reshape(*lead, E)


class _RouterFunction(torch.autograd.Function):
    """Router scores with gradients: forward through libspx; backward as the
    reference's autograd computes it for ``softplus(F.linear(x, W, b))`` in
    BF16 (d logits = bf16(g * sigmoid(logits)) for softplus, then the linear
    layer's input, weight and bias gradients)."""

    @staticmethod
    def forward(ctx, router, hidden_states, *params):
        softplus = router.config.router_score_transform != "identity"
        logits = router._scores(hidden_states, identity=True) if softplus else None
        scores = router._scores(hidden_states, identity=False)
        ctx.save_for_backward(hidden_states, logits, *params)
        ctx.softplus = softplus
        ctx.has_bias = len(params) > 1
        return scores

    @staticmethod
    def backward(ctx, grad):
        x, logits, *params = ctx.saved_tensors
        w = params[0]
        g = grad
        if ctx.softplus:  # F.softplus backward (beta 1, threshold 20)
            z = logits.float()
            g = torch.where(z > 20.0, grad.float(), grad.float() * torch.sigmoid(z)).to(grad.dtype)
        g2 = g.reshape(-1, g.shape[-1])
        x2 = x.reshape(-1, x.shape[-1])
        dx = (g2 @ w).reshape(x.shape) if ctx.needs_input_grad[1] else None
        dw = g2.t() @ x2 if ctx.needs_input_grad[2] else None
        out = [None, dx, dw]
        if ctx.has_bias:
            out.append(g2.sum(0) if ctx.needs_input_grad[3] else None)
        return tuple(out)


class MicroExpertBank(nn.Module):
    """Stacked expert projections, reference layout (experts/bank.py:37-54)."""

    def __init__(self, config) -> None:
        super().__init__()
        config = coerce_config(config)
        self.config = config
        e, d, i = config.num_experts, config.d_model, config.resolved_inter_dim
        std = config.initializer_range
        self.gate_proj = nn.Parameter(torch.randn(e, d, i) * std)
        self.up_proj = nn.Parameter(torch.randn(e, d, i) * std)
        self.down_proj = nn.Parameter(torch.randn(e, i, d) * std)

        object.__setattr__(self, "_offload", None)  # PagedExpertCache while offloaded

    @property
    def num_experts(self) -> int:
        return self.config.num_experts

    @property
    def parameters_per_expert(self) -> int:
        return self.gate_proj[0].numel() + self.up_proj[0].numel() + self.down_proj[0].numel()

    # ---- expert offload (bank.py:95-407); the cache itself is spalmer_b200.offload.PagedExpertCache
    @property
    def expert_offload_enabled(self) -> bool:
        return self._offload is not None

    @property
    def expert_paging_enabled(self) -> bool:
        return self._offload is not None and self._offload.paging

    @property
    def expert_cache_capacity(self) -> int | None:
        return None if self._offload is None else self._offload.capacity

    @property
    def expert_offload_counters(self) -> tuple[int, int, int, int]:
        """Stage operations, transferred rows, evicted rows, transferred bytes
        (bytes of the BF16 masters, as the reference counts them)."""

        return (0, 0, 0, 0) if self._offload is None else tuple(self._offload.policy.counters)

    @property
    def cached_expert_ids(self) -> tuple[int, ...]:
        return () if self._offload is None else self._offload.policy.cached_ids

    @property
    def expert_cache_device(self) -> torch.device | None:
        return None if self._offload is None else self._offload.target

    @property
    def expert_master_device(self) -> torch.device:
        devices = {p.device for p in self.parameters(recurse=False)}
        if len(devices) != 1:
            raise RuntimeError(f"expert master projections span devices: {sorted(map(str, devices))}")
        return next(iter(devices))

    @property
    def expert_master_bytes(self) -> int:
        return sum(p.numel() * p.element_size() for p in self.parameters(recurse=False))

    @property
    def expert_masters_pinned(self) -> bool:
        params = tuple(self.parameters(recurse=False))
        return bool(params) and all(p.is_pinned() for p in params)

    @property
    def expert_cache_bytes(self) -> int:
        """Physical bytes of the device cache (every slot, packed layouts)."""

        return 0 if self._offload is None else self._offload.cache_bytes

    @property
    def expert_cache_index_bytes(self) -> int:
        """Bytes of one expert-to-slot table ([E] int32) handed to the kernels."""

        return 0 if self._offload is None else 4 * self.num_experts

    def _apply(self, fn, recurse: bool = True):
        # Offloaded masters stay on the CPU when the module around them moves.
        if self._offload is not None:
            return self
        return super()._apply(fn, recurse=recurse)

    @torch.no_grad()
    def _prepare_expert_offload(self, target_device: torch.device, *, capacity: int, non_blocking: bool,
                                pin_memory: bool, paging: bool = False) -> None:
        """Keep the masters on the CPU and prepare an empty device cache (bank.py:195-238)."""

        from spalmer_b200.offload import PagedExpertCache

        if self.training:
            raise RuntimeError("expert offload is inference-only; put the model in eval mode first")
        if self._offload is not None:
            raise RuntimeError("expert offload is already enabled for this bank")
        if not 1 <= capacity <= self.num_experts:
            raise ValueError(f"expert cache capacity must lie in [1, {self.num_experts}]; got {capacity}")
        self.to(device="cpu")
        if pin_memory:
            for p in self.parameters(recurse=False):
                try:
                    p.data = p.detach().pin_memory()
                except RuntimeError:
                    break  # page locking is an optimisation; telemetry reports what happened
        object.__setattr__(self, "_offload", PagedExpertCache(self, torch.device(target_device), capacity,
                                                              non_blocking=non_blocking, paging=paging))

    @torch.no_grad()
    def _stage_expert_rows(self, expert_ids: tuple[int, ...], *, force: bool = False) -> tuple[int, int, int]:
        """Stage exactly ``expert_ids`` (sorted, unique); returns rows in,
        rows out, bytes in (bank.py:241-332)."""

        cache = self._offload
        if cache is None:
            raise RuntimeError("expert offload has not been prepared for this bank")
        if any(p.device.type != "cpu" for p in self.parameters(recurse=False)):
            raise RuntimeError("offloaded expert master parameters must remain on CPU")
        plan = cache.policy.plan_rows(tuple(expert_ids), force=force)
        if plan is None:
            return 0, 0, 0
        cache.stage_now(plan)
        return len(plan.incoming), len(plan.evicted), len(plan.incoming) * cache.policy.bytes_per_row

    @torch.no_grad()
    def _stage_execution_page(self, required_ids: tuple[int, ...]) -> None:
        """Stage the required ids and keep recent rows in spare slots (bank.py:341-365)."""

        cache = self._offload
        if cache is None or not cache.paging:
            raise RuntimeError("layer-local expert paging is not enabled")
        plan, lru = cache.policy.plan_page(required_ids)
        cache.stage_now(plan, lru)

    def _clear_expert_offload(self) -> None:
        object.__setattr__(self, "_offload", None)

    # ---- the bank seam: execute given routing pairs (bank.py:593-646)
    def execute_routing(self, hidden_states: Tensor, token_index: Tensor, expert_index: Tensor,
                        routing_weights: Tensor, promoted_mask: Tensor | None = None,
                        resident_ids: Tensor | None = None) -> Tensor:
        """Execute only the selected (token, expert) pairs and return the
        ``[num_tokens, d_model]`` weighted combination of their updates
        (``MicroExpertBank.execute_routing``, experts/bank.py:593-646).

        The pairs' rows are gathered (``spx_gather_rows``), run through the
        grouped tcgen05 expert GEMMs unweighted in a stable per-expert order
        (``spx_experts_forward``; experts whose precision pair under
        ``promoted_mask`` is MXFP8/NVFP4 run in that lane), and each token's
        pairs are summed as ``bf16(bf16(out) * w)`` in pair order with an FP32
        accumulator (``spx_combine``), where the reference index_adds in BF16.
        With ``resident_ids`` the grouped executor runs only the groups of
        those experts (bank.py:725-731): pairs of other experts contribute
        nothing; the loop executor runs every pair.  One host read (the
        largest number of pairs of one token) sizes the combine's slot table;
        the reference's grouped path reads its counts on the host as well.
        """

        if self._offload is not None:
            raise RuntimeError("execute_routing on an offloaded bank: run the layer forward, which pages experts")
        e, d = self.num_experts, self.config.d_model
        if hidden_states.ndim != 2 or hidden_states.shape[1] != d:
            raise ValueError(f"hidden_states must be [num_tokens, {d}], got {tuple(hidden_states.shape)}")
        device = hidden_states.device
        if device.type != "cuda":
            raise RuntimeError(f"the B200 expert bank executes CUDA tensors; hidden states are on {device}")
        weight_fmt = self.config.expert_weight_format
        if weight_fmt == "float32":
            raise NativeExpertPrecisionError("no B200 kernel for float32 experts; emulation is prohibited")
        if hidden_states.dtype != torch.bfloat16:
            raise RuntimeError(
                f"{weight_fmt}/{self.config.expert_activation_format} expert execution requires "
                f"torch.bfloat16 hidden states, got {hidden_states.dtype}"
            )
        P = token_index.numel()
        if token_index.shape != (P,) or expert_index.shape != (P,) or routing_weights.shape != (P,):
            raise ValueError("token_index, expert_index and routing_weights must be matching 1-D tensors")
        N = hidden_states.shape[0]
        if resident_ids is not None and self.config.expert_execution == "grouped" and P > 0:
            keep = torch.isin(expert_index.to(device), resident_ids.to(device=device, dtype=torch.long))
            token_index, expert_index, routing_weights = token_index[keep], expert_index[keep], routing_weights[keep]
            P = token_index.numel()
        out = torch.zeros(N, d, dtype=torch.bfloat16, device=device)
        if P == 0 or N == 0:
            return out
        lib = _lib.load()
        stream = torch.cuda.current_stream(device).cuda_stream
        x = hidden_states.contiguous()
        tok32 = token_index.to(device=device, dtype=torch.int32).contiguous()
        rows = torch.empty(P, d, dtype=torch.bfloat16, device=device)
        _lib.check(lib.spx_gather_rows(x.data_ptr(), d, tok32.data_ptr(), 1, P, d, rows.data_ptr(), d, stream),
                   "spx_gather_rows")
        dims = self._pair_dims(P)
        pw = self._packed_experts(device, dims)
        lanes = self._lanes_of(promoted_mask, device)
        if lanes is not None:
            mx = pw["mx"]
            pw["weights"].expert_lane_mxfp8 = lanes.data_ptr()
            pw["weights"].expert_w1_mx = _lib.ptr(mx["expert_w1_mx"])
            pw["weights"].expert_w1_mx_scales = _lib.ptr(mx["expert_w1_mx_scales"])
            pw["weights"].expert_w2_mx = _lib.ptr(mx["expert_w2_mx"])
            pw["weights"].expert_w2_mx_scales = _lib.ptr(mx["expert_w2_mx_scales"])
            pw["weights"].expert_nvfp4_amax = _lib.ptr(mx.get("expert_nvfp4_amax"))
        else:
            pw["weights"].expert_lane_mxfp8 = None
        nbytes = _lib.ctypes.c_size_t()
        _lib.check(lib.spx_layer_sizes(dims, nbytes, None), "spx_layer_sizes")
        ws = torch.zeros(nbytes.value, dtype=torch.uint8, device=device)
        ids = expert_index.to(device=device, dtype=torch.int64).contiguous()
        y = torch.empty(P, d, dtype=torch.bfloat16, device=device)
        _lib.check(lib.spx_experts_forward(dims, pw["weights"], rows.data_ptr(), ids.data_ptr(), y.data_ptr(),
                                           ws.data_ptr(), stream), "spx_experts_forward")
        status = _lib.ctypes.c_int(0)
        _lib.check(lib.spx_workspace_status(ws.data_ptr(), status, 1, stream), "spx_workspace_status")
        if status.value != 0:
            raise RuntimeError(f"expert kernels reported device status {status.value} (expert id out of range?)")
        # per token, its pairs in pair order: slot table [N, slots], -1 = empty
        tok = token_index.to(device=device, dtype=torch.int64)
        counts = torch.bincount(tok, minlength=N)
        slots = int(counts.max())
        perm = torch.argsort(tok, stable=True)
        starts = torch.cumsum(counts, 0) - counts
        slot = torch.arange(P, device=device) - starts[tok[perm]]
        table = torch.full((N * slots,), -1, dtype=torch.int32, device=device)
        table[tok[perm] * slots + slot] = perm.to(torch.int32)
        wtab = torch.zeros(N * slots, dtype=torch.bfloat16, device=device)
        wtab[tok[perm] * slots + slot] = routing_weights.to(device=device, dtype=torch.bfloat16)[perm]
        table, wtab = table.view(N, slots), wtab.view(N, slots)
        base = None
        for j0 in range(0, slots, _MAX_COMBINE_SLOTS):  # the combine adds up to 20 slots per pass
            j1 = min(slots, j0 + _MAX_COMBINE_SLOTS)
            t_part, w_part = table[:, j0:j1].contiguous(), wtab[:, j0:j1].contiguous()
            res = torch.empty(N, d, dtype=torch.bfloat16, device=device)
            _lib.check(lib.spx_combine(y.data_ptr(), t_part.data_ptr(), w_part.data_ptr(), _lib.ptr(base), N, d,
                                       j1 - j0, res.data_ptr(), stream), "spx_combine")
            base = res
        return base

    def _pair_dims(self, pairs: int) -> _lib.LayerDims:
        dims = layer_dims(self.config, pairs, 1)
        dims.shared_dim = 0
        return dims

    def _lanes_of(self, promoted_mask: Tensor | None, device: torch.device) -> Tensor | None:
        unpromoted, promoted = _lane_of(self.config, False), _lane_of(self.config, True)
        if unpromoted == 0 and (promoted == 0 or promoted_mask is None):
            return None
        if promoted_mask is None:
            return torch.ones(self.num_experts, dtype=torch.uint8, device=device)
        if promoted_mask.shape != (self.num_experts,):
            raise ValueError(f"promoted_mask must have shape ({self.num_experts},)")
        m = promoted_mask.to(device=device, dtype=torch.bool)
        return torch.where(m, int(promoted != 0), int(unpromoted != 0)).to(torch.uint8).contiguous()

    def _packed_experts(self, device: torch.device, dims: _lib.LayerDims) -> dict:
        """Kernel layouts of the expert masters for the bank seam (one cache
        entry per batch class, invalidated when a master changes)."""

        small = dims.tokens <= SMALL_BATCH_TOKENS
        masters = (self.gate_proj, self.up_proj, self.down_proj)
        key = (device, small, dims.mxfp8_lane) + tuple((t.data_ptr(), t._version) for t in masters)
        cache = self.__dict__.setdefault("_seam_pack", {})
        hit = cache.get(small)
        if hit is not None and hit["key"] == key:
            return hit
        for t in masters:
            if t.device != device or t.dtype != torch.bfloat16:
                raise RuntimeError(f"expert masters must be BF16 on {device}; got {t.dtype} on {t.device}")
        lib = _lib.load()
        sizes = _lib.PackedSizes()
        _lib.check(lib.spx_layer_sizes(dims, None, sizes), "spx_layer_sizes")
        stream = torch.cuda.current_stream(device).cuda_stream
        gate, up, down = (t.detach().contiguous() for t in masters)
        dummy_router = torch.zeros(self.num_experts, self.config.d_model, dtype=torch.bfloat16, device=device)
        router_out = torch.empty(max(1, sizes.router_weight), dtype=torch.int16, device=device)
        w1 = torch.empty(max(1, sizes.expert_w1), dtype=torch.int16, device=device)
        w2 = torch.empty(max(1, sizes.expert_w2), dtype=torch.int16, device=device)
        src = _lib.ReferenceWeights(router_weight=dummy_router.data_ptr(), gate_proj=gate.data_ptr(),
                                    up_proj=up.data_ptr(), down_proj=down.data_ptr())
        _lib.check(lib.spx_pack_weights(dims, src, router_out.data_ptr(), w1.data_ptr(), w2.data_ptr(), None, None,
                                        stream), "spx_pack_weights (experts)")
        mx = {}
        if dims.mxfp8_lane:
            mx = pack_lowp_experts(dims, src, sizes, lambda n: torch.empty(n, dtype=torch.uint8, device=device),
                                   stream)
        weights = _lib.PackedWeights(expert_w1=w1.data_ptr(), expert_w2=w2.data_ptr())
        entry = {"key": key, "weights": weights, "mx": mx, "keep": (gate, up, down, dummy_router, router_out, w1, w2)}
        cache[small] = entry
        return entry


class SwiGLU(nn.Module):
    """Shared gated MLP parameters (nn/ffn.py:9-25)."""

    def __init__(self, d_model: int, hidden_size: int, *, initializer_range: float | None = None):
        super().__init__()
        if d_model <= 0 or hidden_size <= 0:
            raise ValueError("d_model and hidden_size must be positive")
        self.gate_projection = nn.Linear(d_model, hidden_size, bias=False)
        self.up_projection = nn.Linear(d_model, hidden_size, bias=False)
        self.down_projection = nn.Linear(hidden_size, d_model, bias=False)
        if initializer_range is not None:
            for linear in (self.gate_projection, self.up_projection, self.down_projection):
                nn.init.normal_(linear.weight, mean=0.0, std=initializer_range)

    @property
    def parameter_count(self) -> int:
        return sum(p.numel() for p in self.parameters())


class ExpertPotentiationController(nn.Module):
    """Checkpoint-visible promotion state (experts/potentiation.py:24-47).

    The B200 layer consumes ``promoted_mask``; the EMA update policy of the
    reference controller is outside this hot path.
    """

    def __init__(self, config) -> None:
        super().__init__()
        config = coerce_config(config)
        self.config = config
        shape = (config.num_experts,)
        self.register_buffer("utilization_ema", torch.zeros(shape, dtype=torch.float32))
        self.register_buffer("attributed_nll_ema", torch.zeros(shape, dtype=torch.float32))
        self.register_buffer("quantization_error_ema", torch.zeros(shape, dtype=torch.float32))
        self.register_buffer("promoted_mask", torch.zeros(shape, dtype=torch.bool))
        self.register_buffer("observations", torch.zeros((), dtype=torch.long))
        self.register_buffer("last_change", torch.zeros((), dtype=torch.long))

    def _apply(self, fn, recurse: bool = True):
        super()._apply(fn, recurse)
        for name in ("utilization_ema", "attributed_nll_ema", "quantization_error_ema"):
            self._buffers[name] = self._buffers[name].float()
        return self


class ExpertResidency(nn.Module):
    """Resident expert set shared by all layers (experts/residency.py:59-215 subset)."""

    def __init__(self, config) -> None:
        super().__init__()
        config = coerce_config(config)
        self.config = config
        self._ids: tuple[int, ...] = tuple(range(config.num_experts))
        self._active_experts_override: int | None = None
        self.register_buffer("resident_mask", torch.ones(config.num_experts, dtype=torch.bool), persistent=False)
        self.register_buffer(
            "resident_ids", torch.arange(config.num_experts, dtype=torch.long), persistent=False
        )

    @property
    def num_experts(self) -> int:
        return self.config.num_experts

    @property
    def ids(self) -> tuple[int, ...]:
        return self._ids

    @property
    def size(self) -> int:
        return len(self._ids)

    @property
    def is_full(self) -> bool:
        return len(self._ids) == self.num_experts

    @property
    def active_experts(self) -> int:
        if self._active_experts_override is not None:
            return self._active_experts_override
        return self.config.active_experts

    @property
    def active_experts_override(self) -> int | None:
        return self._active_experts_override

    @property
    def max_active_experts(self) -> int:
        return min(self.config.max_active_experts, self.num_experts)

    def set_active_experts(self, count: int | None) -> None:
        if count is not None and not self.config.min_active_experts <= count <= self.max_active_experts:
            raise ValueError(
                f"active_experts must be in [{self.config.min_active_experts}, {self.max_active_experts}]; "
                f"got {count}"
            )
        effective = self.config.active_experts if count is None else count
        if effective > self.size:
            raise ValueError(f"per-token top-{effective} cannot be served by only {self.size} resident experts")
        self._active_experts_override = count

    def set(self, ids) -> tuple[int, ...]:
        unique = tuple(sorted({int(e) for e in ids}))
        if not unique:
            raise ValueError("the resident set cannot be empty")
        if unique[0] < 0 or unique[-1] >= self.num_experts:
            raise ValueError(f"expert ids must be in [0, {self.num_experts})")
        if len(unique) < self.active_experts:
            raise ValueError(f"{len(unique)} resident experts cannot serve a per-token top-{self.active_experts}")
        if len(unique) > self.config.resident_cap and len(unique) != self.num_experts:
            raise ValueError(f"resident set of {len(unique)} exceeds the cap {self.config.resident_cap}")
        self._ids = unique
        mask = torch.zeros(self.num_experts, dtype=torch.bool, device=self.resident_mask.device)
        mask[list(unique)] = True
        self.resident_mask.copy_(mask)
        self.resident_ids = torch.tensor(unique, dtype=torch.long, device=self.resident_mask.device)
        return unique


# ---------------------------------------------------------------- device caches

_SOFTPLUS: dict[torch.device, Tensor] = {}


def softplus_table(device: torch.device) -> Tensor:
    """The BF16 softplus table of ``device`` (computed once by a libspx kernel)."""

    table = _SOFTPLUS.get(device)
    if table is None:
        lib = _lib.load()
        table = torch.empty(65536, dtype=torch.int16, device=device)
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(lib.spx_softplus_table(table.data_ptr(), stream), "spx_softplus_table")
        _SOFTPLUS[device] = table
    return table


# Batches of at most this many tokens use the decode tile shapes (kSmallBatchTokens in libspx).
SMALL_BATCH_TOKENS = 256
# Slots one spx_combine pass adds per token (kMaxTopK in libspx).
_MAX_COMBINE_SLOTS = 20


def layer_dims(config: MicroExpertsConfig, tokens: int, top_k: int) -> _lib.LayerDims:
    return _lib.LayerDims(
        tokens=tokens,
        d_model=config.d_model,
        num_experts=config.num_experts,
        inter_dim=config.resolved_inter_dim,
        shared_dim=config.resolved_shared_inter_dim,
        top_k=top_k,
        score_transform=0 if config.router_score_transform == "softplus" else 1,
        execution_loop=1 if config.expert_execution == "loop" else 0,
        mxfp8_lane=lowp_lane(config),
    )


# Precision pairs with a B200 kernel lane: 0 = BF16 grouped GEMM, 1 = MXFP8
# block-scaled grouped GEMM, 2 = NVFP4 block-scaled grouped GEMM.
_LANES = {("bfloat16", "bfloat16"): 0, ("mxfp8", "mxfp8"): 1, ("nvfp4", "nvfp4"): 2}
LOWP_ARRAYS = ("expert_w1_mx", "expert_w1_mx_scales", "expert_w2_mx", "expert_w2_mx_scales")


def execution_pair(config: MicroExpertsConfig, promoted: bool) -> tuple[str, str]:
    """``MicroExpertBank._execution_pair`` (experts/bank.py:462-475)."""

    if not promoted:
        return config.expert_weight_format, config.expert_activation_format
    fmt = config.expert_promotion_format
    if fmt in {"bfloat16", "mxfp8", "float32"}:
        return fmt, fmt
    raise RuntimeError(f"no native promotion kernel for {fmt!r}")


def _lane_of(config: MicroExpertsConfig, promoted: bool) -> int:
    pair = execution_pair(config, promoted)
    lane = _LANES.get(pair)
    if lane is None:
        raise NativeExpertPrecisionError(
            f"no B200 kernel for {pair[0]}/{pair[1]} experts; emulation is prohibited"
        )
    return lane


def lowp_lane(config: MicroExpertsConfig) -> int:
    """The layer's low-precision kernel lane: 0 none, 1 MXFP8, 2 NVFP4.  A layer
    runs at most one of them beside BF16 (NVFP4 experts promoted to MXFP8 have
    no kernel here)."""

    lanes = {_lane_of(config, False), _lane_of(config, True)} - {0}
    if len(lanes) > 1:
        raise NativeExpertPrecisionError(
            "no B200 kernel for NVFP4 experts with an MXFP8 promotion lane; promote to bfloat16"
        )
    return lanes.pop() if lanes else 0


def uses_mxfp8_lane(config: MicroExpertsConfig) -> bool:
    """True when some expert can execute a low-precision (MXFP8 or NVFP4) pair."""

    return lowp_lane(config) != 0


def pack_lowp_experts(dims: _lib.LayerDims, src: _lib.ReferenceWeights, sizes: _lib.PackedSizes,
                      alloc, stream: int) -> dict[str, Tensor]:
    """The low-precision copies of the expert masters for ``dims`` (MXFP8 or
    NVFP4 by ``dims.mxfp8_lane``); ``alloc(nbytes)`` returns a uint8 device tensor."""

    lib = _lib.load()
    out = {name: alloc(max(16, getattr(sizes, name))) for name in LOWP_ARRAYS}
    ptrs = [_lib.ptr(out[name]) for name in LOWP_ARRAYS]
    if dims.mxfp8_lane == 2:
        out["expert_nvfp4_amax"] = alloc(max(16, sizes.expert_nvfp4_amax))
        _lib.check(lib.spx_pack_weights_nvfp4(dims, src, *ptrs, _lib.ptr(out["expert_nvfp4_amax"]), stream),
                   "spx_pack_weights_nvfp4")
    else:
        _lib.check(lib.spx_pack_weights_mxfp8(dims, src, *ptrs, stream), "spx_pack_weights_mxfp8")
    return out


def _bits(t: Tensor) -> Tensor:
    return t.detach().contiguous()


# expert_weight_format -> spx_expert_quant_error's weight_format
_QUANT_ERROR_FORMATS = {"mxfp8": 1, "nvfp4": 2}


class B200MicroExpertChannelMixer(nn.Module):
    """Shared SwiGLU plus routed micro-experts on B200 (experts/mixer.py:38-241)."""

    def __init__(self, config, *, router: SurpriseRouter | None = None,
                 potentiation_controller: ExpertPotentiationController | None = None,
                 residency: ExpertResidency | None = None) -> None:
        super().__init__()
        config = coerce_config(config)
        if router is not None:
            if router.num_experts != config.num_experts:
                raise ValueError(
                    f"shared router serves {router.num_experts} experts; this bank has {config.num_experts}"
                )
            if router.num_features != config.d_model:
                raise ValueError(
                    f"shared router expects width {router.num_features}; this layer has {config.d_model}"
                )
        self.config = config
        self.router = router if router is not None else SurpriseRouter(config)
        self.experts = MicroExpertBank(config)
        width = config.resolved_shared_inter_dim
        self.shared = SwiGLU(config.d_model, width, initializer_range=config.initializer_range) if width > 0 else None
        if potentiation_controller is None:
            self._owned_potentiation_controller = ExpertPotentiationController(config)
            potentiation_controller = self._owned_potentiation_controller
        elif coerce_config(potentiation_controller.config) != config:
            raise ValueError("potentiation controller configuration does not match this bank")
        if residency is None:
            self._owned_residency = ExpertResidency(config)
            residency = self._owned_residency
        elif coerce_config(residency.config) != config:
            raise ValueError("residency configuration does not match this bank")
        object.__setattr__(self, "_potentiation_controller_ref", ref(potentiation_controller))
        object.__setattr__(self, "_residency_ref", ref(residency))
        object.__setattr__(self, "_pack_cache", {})
        object.__setattr__(self, "_quant_error_cache", None)
        object.__setattr__(self, "_lane_cache", None)
        object.__setattr__(self, "_ws_cache", {})
        object.__setattr__(self, "_stage_event_array", None)

    def record_stage_events(self, events: list | None) -> None:
        """Record ``SPX_STAGE_EVENTS`` torch CUDA events at the kernel-stage
        boundaries of every following forward (``None`` switches it off)."""

        if events is None:
            object.__setattr__(self, "_stage_event_array", None)
            return
        if len(events) != _lib.STAGE_EVENTS:
            raise ValueError(f"need {_lib.STAGE_EVENTS} events")
        handles = []
        for ev in events:
            if ev.cuda_event == 0:  # torch creates the event lazily on first record
                ev.record()
            handles.append(ev.cuda_event)
        array = (_lib.ctypes.c_void_p * len(handles))(*handles)
        object.__setattr__(self, "_stage_event_array", array)

    # ---- reference-compatible properties
    @property
    def potentiation_controller(self) -> ExpertPotentiationController:
        controller = self._potentiation_controller_ref()
        if controller is None:
            raise RuntimeError("the shared potentiation controller no longer exists")
        return controller

    @property
    def residency(self) -> ExpertResidency:
        residency = self._residency_ref()
        if residency is None:
            raise RuntimeError("the shared expert residency no longer exists")
        return residency

    @property
    def active_experts(self) -> int:
        return self.residency.active_experts

    @property
    def active_experts_override(self) -> int | None:
        return self.residency.active_experts_override

    @property
    def max_active_experts(self) -> int:
        return self.residency.max_active_experts

    def set_active_experts(self, count: int | None) -> None:
        self.residency.set_active_experts(count)

    @property
    def has_shared_path(self) -> bool:
        return self.shared is not None

    # ---- derived caches
    def _weight_tensors(self) -> dict[str, Tensor | None]:
        s = self.shared
        return {
            "router_weight": self.router.proj.weight,
            "router_bias": self.router.proj.bias,
            "gate_proj": self.experts.gate_proj,
            "up_proj": self.experts.up_proj,
            "down_proj": self.experts.down_proj,
            "shared_gate": None if s is None else s.gate_projection.weight,
            "shared_up": None if s is None else s.up_projection.weight,
            "shared_down": None if s is None else s.down_projection.weight,
        }

    def _packed(self, device: torch.device, tokens: int, top_k: int) -> dict[str, Tensor | None]:
        """Kernel layouts of the weights, one cache entry per batch class
        (decode-sized batches of <= 256 tokens use narrower GEMM1 chunks).
        With expert offload the expert bank is packed by its cache instead."""

        tensors = self._weight_tensors()
        offloaded = self.experts.expert_offload_enabled
        if offloaded:
            for name in ("gate_proj", "up_proj", "down_proj"):
                tensors[name] = None
        key = (device, offloaded) + tuple(
            (None if t is None else (t.data_ptr(), t._version, t.dtype)) for t in tensors.values()
        )
        batch_class = tokens <= SMALL_BATCH_TOKENS
        cache = self._pack_cache.get(batch_class)
        if cache is not None and cache[0] == key:
            return cache[1]
        for name, t in tensors.items():
            if t is None:
                continue
            if t.device != device:
                raise RuntimeError(f"parameter {name} is on {t.device}, hidden states on {device}")
            if t.dtype != torch.bfloat16:
                raise RuntimeError(
                    f"the B200 layer executes BF16 weights; {name} is {t.dtype} (cast the module with .to(torch.bfloat16))"
                )
        lib = _lib.load()
        dims = layer_dims(self.config, tokens, top_k)
        sizes = _lib.PackedSizes()
        _lib.check(lib.spx_layer_sizes(dims, None, sizes), "spx_layer_sizes")
        bits = {n: (None if t is None else _bits(t)) for n, t in tensors.items()}
        empty = lambda n: torch.empty(max(1, n), dtype=torch.int16, device=device)  # noqa: E731
        packed = {
            "router_weight": empty(sizes.router_weight),
            "expert_w1": None if offloaded else empty(sizes.expert_w1),
            "expert_w2": None if offloaded else empty(sizes.expert_w2),
            "shared_w1": empty(sizes.shared_w1) if sizes.shared_w1 else None,
            "shared_w2": empty(sizes.shared_w2) if sizes.shared_w2 else None,
            "router_bias": bits["router_bias"],
        }
        src = _lib.ReferenceWeights(*(_lib.ptr(bits[n]) for n in (
            "router_weight", "router_bias", "gate_proj", "up_proj", "down_proj",
            "shared_gate", "shared_up", "shared_down")))
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(
            lib.spx_pack_weights(
                dims, src, _lib.ptr(packed["router_weight"]), _lib.ptr(packed["expert_w1"]),
                _lib.ptr(packed["expert_w2"]), _lib.ptr(packed["shared_w1"]), _lib.ptr(packed["shared_w2"]),
                stream,
            ),
            "spx_pack_weights",
        )
        if dims.mxfp8_lane and not offloaded:
            packed.update(pack_lowp_experts(
                dims, src, sizes, lambda n: torch.empty(n, dtype=torch.uint8, device=device), stream))
        packed["_keepalive"] = bits
        self._pack_cache[batch_class] = (key, packed)
        return packed

    def _quant_error(self, device: torch.device) -> Tensor | None:
        """Reconstruction error of every expert's low-precision copies
        (``MicroExpertBank.quantization_error``, experts/bank.py:526-592), an
        [E] float tensor computed on the device by ``spx_expert_quant_error``
        whenever the masters change; each forward's dispatch reports it for
        the selected experts.  None for bfloat16 / float32 expert weights (the
        reported errors are zeros).  With expert offload the paged cache
        computes it while packing its host bank."""

        fmt = _QUANT_ERROR_FORMATS.get(self.config.expert_weight_format)
        if fmt is None:
            return None
        if self.experts.expert_offload_enabled:
            cache = self.experts._offload
            cache.ensure_packed()
            return cache.quant_error
        ex = self.experts
        masters = (ex.gate_proj, ex.up_proj, ex.down_proj)
        key = (device,) + tuple((t.data_ptr(), t._version) for t in masters)
        cached = self._quant_error_cache
        if cached is not None and cached[0] == key:
            return cached[1]
        out = torch.empty(self.config.num_experts, dtype=torch.float32, device=device)
        bits = [_bits(t) for t in masters]
        src = _lib.ReferenceWeights(gate_proj=bits[0].data_ptr(), up_proj=bits[1].data_ptr(),
                                    down_proj=bits[2].data_ptr())
        dims = layer_dims(self.config, 1, self.active_experts)
        _lib.check(_lib.load().spx_expert_quant_error(dims, src, fmt, out.data_ptr(),
                                                      torch.cuda.current_stream(device).cuda_stream),
                   "spx_expert_quant_error")
        object.__setattr__(self, "_quant_error_cache", (key, out))
        return out

    def _lanes(self, device: torch.device) -> Tensor | None:
        """Per-expert kernel lane (uint8 [E], 1 = the layer's low-precision lane,
        MXFP8 or NVFP4) from the promotion mask.

        ``MicroExpertBank._execution_pair`` (experts/bank.py:462-475) decides each
        expert's precision pair from ``promoted_mask``; the lane tensor is built on
        the device (no host read of the mask) and cached on the mask's version.
        None when every expert runs BF16.
        """

        config = self.config
        unpromoted, promoted = _lane_of(config, False), _lane_of(config, True)
        if unpromoted == 0 and promoted == 0:
            return None
        mask = self.potentiation_controller.promoted_mask
        key = (device, mask.data_ptr(), mask._version)
        cached = self._lane_cache
        if cached is not None and cached[0] == key:
            return cached[1]
        m = mask.detach().to(device=device, dtype=torch.bool)
        # the kernels take 1 = the layer's low-precision lane (MXFP8 or NVFP4), 0 = BF16
        lanes = torch.where(m, int(promoted != 0), int(unpromoted != 0)).to(torch.uint8).contiguous()
        object.__setattr__(self, "_lane_cache", (key, lanes))
        return lanes

    def _workspace(self, device: torch.device, dims: _lib.LayerDims) -> Tensor:
        lib = _lib.load()
        nbytes = _lib.ctypes.c_size_t()
        _lib.check(lib.spx_layer_sizes(dims, nbytes, None), "spx_layer_sizes")
        key = (device, nbytes.value)
        ws = self._ws_cache.get(key)
        if ws is None:
            self._ws_cache.clear()
            ws = torch.zeros(nbytes.value, dtype=torch.uint8, device=device)
            self._ws_cache[key] = ws
        return ws

    def device_status(self, clear: bool = True) -> int:
        """Device status word of the last workspace (synchronises); 0 means no kernel error."""

        lib = _lib.load()
        for (device, _), ws in self._ws_cache.items():
            value = _lib.ctypes.c_int(0)
            stream = torch.cuda.current_stream(device).cuda_stream
            _lib.check(lib.spx_workspace_status(ws.data_ptr(), value, int(clear), stream), "spx_workspace_status")
            return value.value
        return 0

    # ---- forward
    def forward(self, hidden_states: Tensor, *, state: Any = None,
                router_logits: Tensor | None = None) -> ChannelMixerOutput:
        """Run the layer; see ``experts/mixer.py:145-241`` for the contract.

        ``router_logits`` (optional, ``[batch, seq, experts]`` BF16) replaces
        the router GEMM output; it exists to check the routing contract
        "bit-exact given identical logits".
        """

        if hidden_states.ndim != 3:
            raise ValueError(
                f"hidden_states must have shape [batch, seq, d_model]; got {tuple(hidden_states.shape)}"
            )
        config = self.config
        if hidden_states.shape[-1] != config.d_model:
            raise ValueError(f"expected trailing dimension {config.d_model}; got {hidden_states.shape[-1]}")
        # Expert offload is inference-only (offload.py:15-18): its forward records no graph.
        if torch.is_grad_enabled() and not self.experts.expert_offload_enabled and (
            hidden_states.requires_grad or any(p.requires_grad for p in self.parameters())
        ):
            if router_logits is not None:
                raise ValueError("router_logits injection checks the forward only; run it without gradients")
            return self._forward_autograd(hidden_states)
        return self._forward_native(hidden_states, router_logits)

    def _training_saves(self, hidden_states: Tensor) -> tuple | None:
        """Buffers for the activations the backward would otherwise recompute,
        when this layer's native backward can take them (BF16 experts on the
        device, d_model % 64 == 0, prefill-sized batches): (the hidden rows and
        the gate | up pre-activations of the expert GEMM1 in dispatch order, the
        router logits of softplus scores or None, the shared SwiGLU's gate | up
        pre-activations with their chunk width or None)."""
        config = self.config
        batch, seq_len, d = hidden_states.shape
        k = self.active_experts
        P = batch * seq_len * k
        if (self._lanes(hidden_states.device) is not None or self.experts.expert_offload_enabled or d % 64
                or config.resolved_inter_dim % 8 or P <= 1024):
            return None
        cols = _lib.ctypes.c_int64()
        lib = _lib.load()
        _lib.check(lib.spx_layer_saved_gu_cols(layer_dims(config, batch * seq_len, k), cols),
                   "spx_layer_saved_gu_cols")
        device = hidden_states.device
        T = batch * seq_len
        logits = None
        if config.router_score_transform == "softplus":
            logits = torch.empty(T, config.num_experts, dtype=torch.bfloat16, device=device)
        shared_gu = None
        if self.shared is not None and _shared_bwd_native(self.shared, hidden_states.reshape(T, d)):
            scols = _lib.ctypes.c_int64()
            chunk = _lib.ctypes.c_int32()
            _lib.check(lib.spx_layer_saved_shared_gu(layer_dims(config, T, k), scols, chunk),
                       "spx_layer_saved_shared_gu")
            if self.shared.gate_projection.weight.shape[0] % chunk.value == 0:  # whole chunks
                shared_gu = (torch.empty(T, scols.value, dtype=torch.bfloat16, device=device), chunk.value)
        return (torch.empty(P, d, dtype=torch.bfloat16, device=device),
                torch.empty(P, cols.value, dtype=torch.bfloat16, device=device), logits, shared_gu)

    def _forward_native(self, hidden_states: Tensor, router_logits: Tensor | None,
                        block: tuple[Tensor, float, Tensor] | None = None,
                        saved: tuple | None = None) -> ChannelMixerOutput:
        config = self.config
        if not hidden_states.is_cuda:
            raise RuntimeError("the B200 micro-expert layer requires CUDA hidden states")
        if hidden_states.dtype != torch.bfloat16:
            raise RuntimeError(
                f"{config.expert_weight_format}/{config.expert_activation_format} expert execution requires "
                f"torch.bfloat16 hidden states, got {hidden_states.dtype}"
            )
        lanes = self._lanes(hidden_states.device)
        batch, seq_len, d_model = hidden_states.shape
        tokens = batch * seq_len
        k = self.active_experts
        residency = self.residency
        full_pool = residency.is_full
        if not full_pool and residency.size < k:
            raise ValueError(f"{residency.size} resident experts cannot serve a per-token top-{k}")
        device = hidden_states.device
        E = config.num_experts
        lib = _lib.load()
        dims = layer_dims(config, tokens, k)
        packed = self._packed(device, tokens, k)
        ws = self._workspace(device, dims)
        self._ws_generation = getattr(self, "_ws_generation", 0) + 1  # this call's dispatch now lives in ws
        self._last_forward = (self._ws_generation, ws)
        x = hidden_states.reshape(tokens, d_model).contiguous()
        update = torch.empty(batch, seq_len, d_model, dtype=torch.bfloat16, device=device)
        scores = torch.empty(batch, seq_len, E, dtype=torch.bfloat16, device=device)
        ids = torch.empty(batch, seq_len, k, dtype=torch.long, device=device)
        weights = torch.empty(batch, seq_len, k, dtype=torch.bfloat16, device=device)
        util = torch.empty(E, dtype=torch.float32, device=device)
        stats = torch.empty(6, dtype=torch.long, device=device)
        ratios = torch.empty(2, dtype=torch.float32, device=device)
        aux = torch.empty(1, dtype=torch.bfloat16, device=device)
        quant_error = torch.empty(E, dtype=torch.float32, device=device)
        injected = None
        if router_logits is not None:
            if router_logits.shape != (batch, seq_len, E) or router_logits.dtype != torch.bfloat16:
                raise ValueError("router_logits must be [batch, seq, experts] bfloat16")
            injected = router_logits.contiguous()
        mask = None if full_pool else residency.resident_mask.to(device=device).contiguous()
        lut = softplus_table(device) if config.router_score_transform == "softplus" else None
        pw = _lib.PackedWeights(
            router_weight=_lib.ptr(packed["router_weight"]),
            router_bias=_lib.ptr(packed["router_bias"]),
            expert_w1=_lib.ptr(packed["expert_w1"]),
            expert_w2=_lib.ptr(packed["expert_w2"]),
            shared_w1=_lib.ptr(packed["shared_w1"]),
            shared_w2=_lib.ptr(packed["shared_w2"]),
            softplus_table=_lib.ptr(lut),
            resident_mask=_lib.ptr(mask),
            expert_lane_mxfp8=_lib.ptr(lanes),
            expert_w1_mx=_lib.ptr(packed.get("expert_w1_mx")),
            expert_w1_mx_scales=_lib.ptr(packed.get("expert_w1_mx_scales")),
            expert_w2_mx=_lib.ptr(packed.get("expert_w2_mx")),
            expert_w2_mx_scales=_lib.ptr(packed.get("expert_w2_mx_scales")),
            expert_nvfp4_amax=_lib.ptr(packed.get("expert_nvfp4_amax")),
            expert_quant_error=_lib.ptr(self._quant_error(device)),
        )
        events = self._stage_event_array
        outs = _lib.LayerOutputs(
            update=update.data_ptr(), router_scores=scores.data_ptr(), expert_ids=ids.data_ptr(),
            routing_weights=weights.data_ptr(), expert_utilization=util.data_ptr(),
            group_stats=stats.data_ptr(), group_ratios=ratios.data_ptr(), auxiliary_loss=aux.data_ptr(),
            dispatch_order=None, expert_counts=None, injected_logits=_lib.ptr(injected),
            router_logits=None if saved is None else _lib.ptr(saved[2]),
            stage_events=None if events is None else _lib.ctypes.addressof(events),
            expert_quantization_error=quant_error.data_ptr(),
            saved_x=None if saved is None else saved[0].data_ptr(),
            saved_gu=None if saved is None else saved[1].data_ptr(),
            saved_shared_gu=None if saved is None or saved[3] is None else saved[3][0].data_ptr(),
        )
        stream = torch.cuda.current_stream(device).cuda_stream
        if saved is not None and (self.experts.expert_offload_enabled or block is not None):
            raise RuntimeError("saved training activations come from spx_layer_forward only")
        if self.experts.expert_offload_enabled:
            if block is not None:
                raise RuntimeError("the fused block path needs the expert bank on the device")
            self._run_paged(dims, pw, x, outs, ws, lanes)
        elif block is None:
            _lib.check(lib.spx_layer_forward(dims, pw, x.data_ptr(), outs, ws.data_ptr(), stream),
                       "spx_layer_forward")
        else:
            norm_weight, eps, hidden_out = block
            _lib.check(
                lib.spx_block_channel_forward(dims, pw, norm_weight.data_ptr(), _lib.ctypes.c_float(eps),
                                              x.data_ptr(), outs, hidden_out.data_ptr(), ws.data_ptr(), stream),
                "spx_block_channel_forward",
            )
        controller = self.potentiation_controller
        metrics: dict[str, Any] = {
            "expert_ids": ids,
            "routing_weights": weights,
            "router_scores": scores,
            "expert_utilization": util,
            "expert_quantization_error": quant_error,
            "promoted_experts": controller.promoted_mask.detach().clone(),
            "resident_experts": residency.resident_mask.detach().clone(),
            "expert_paging": self.experts.expert_paging_enabled,
            "routing_full_pool": full_pool,
            "active_experts_per_token": k,
            "num_active_experts": stats[5],
            "expert_execution": config.expert_execution,
            "expert_group_count": stats[0],
            "expert_group_max_load": stats[1],
            "expert_group_real_pairs": stats[2],
            "expert_group_padded_pairs": stats[3],
            "expert_group_padding_amplification": ratios[0],
            "expert_group_global_max_counterfactual_padded_pairs": stats[4],
            "expert_group_global_max_counterfactual_padding_amplification": ratios[1],
        }
        return ChannelMixerOutput(update=update, state=None, auxiliary_loss=aux[0], metrics=metrics)


    def _run_paged(self, dims: _lib.LayerDims, pw: _lib.PackedWeights, x: Tensor, outs: _lib.LayerOutputs,
                   ws: Tensor, lanes: Tensor | None) -> None:
        """The layer with the expert bank behind its device cache
        (bank.py:821-899): route and dispatch, read the per-expert pair counts
        while shared GEMM1 runs, stage and execute the pages, combine."""

        lib = _lib.load()
        cache = self.experts._offload
        device = x.device
        compute = torch.cuda.current_stream(device)
        E = self.config.num_experts
        counts = torch.empty(E, dtype=torch.int32, device=device)
        outs.expert_counts = counts.data_ptr()
        if getattr(self, "_paged_sync", None) is None:
            ev = torch.cuda.Event()
            ev.record(compute)  # creates the event handle
            object.__setattr__(self, "_paged_sync", (ev, torch.cuda.Stream(device)))
        dispatched, side = self._paged_sync
        events = (_lib.ctypes.c_void_p * _lib.STAGE_EVENTS)()
        events[3] = dispatched.cuda_event  # recorded by the library once the dispatch is queued
        outs.stage_events = _lib.ctypes.addressof(events)
        _lib.check(lib.spx_layer_paged_begin(dims, pw, x.data_ptr(), outs, ws.data_ptr(), compute.cuda_stream),
                   "spx_layer_paged_begin")
        outs.stage_events = None
        host_counts = torch.empty(E, dtype=torch.int32, pin_memory=True)
        side.wait_event(dispatched)
        with torch.cuda.stream(side):
            host_counts.copy_(counts, non_blocking=True)
            read = torch.cuda.Event()
            read.record(side)
        counts.record_stream(side)
        read.synchronize()

        def run_chunk(page_slot: Tensor, sm_limit: int) -> None:
            cpw = cache.packed_weights(lanes)
            _lib.check(lib.spx_layer_paged_experts(dims, cpw, cache.capacity, page_slot.data_ptr(), sm_limit,
                                                   x.data_ptr(), ws.data_ptr(), compute.cuda_stream),
                       "spx_layer_paged_experts")

        cache.run_pages(host_counts.numpy(), run_chunk)
        _lib.check(lib.spx_layer_paged_finish(dims, pw, x.data_ptr(), outs, ws.data_ptr(), compute.cuda_stream),
                   "spx_layer_paged_finish")

    # ---- training: forward through the native kernels, backward through spx_layer_backward
    def _trainable(self) -> list[tuple[str, Tensor]]:
        named = dict(self.named_parameters())
        keys = ["router.proj.weight", "router.proj.bias", "experts.gate_proj", "experts.up_proj",
                "experts.down_proj", "shared.gate_projection.weight", "shared.up_projection.weight",
                "shared.down_projection.weight"]
        return [(k, named[k]) for k in keys if k in named]

    def _forward_autograd(self, hidden_states: Tensor) -> ChannelMixerOutput:
        if not hidden_states.is_cuda:
            raise RuntimeError("the B200 micro-expert layer requires CUDA hidden states")
        lanes = self._lanes(hidden_states.device)
        if lanes is not None and bool(lanes.any()):
            raise NativeExpertPrecisionError(
                "provider spx_sm100_grouped has no backward for low-precision (mxfp8/nvfp4) experts; "
                "train with BF16 experts"
            )
        named = self._trainable()
        holder: dict[str, Any] = {}
        update, aux, scores = _LayerFunction.apply(self, holder, [k for k, _ in named], hidden_states,
                                                   *[p for _, p in named])
        metrics = dict(holder["metrics"])
        metrics["router_scores"] = scores
        return ChannelMixerOutput(update=update, state=None, auxiliary_loss=aux, metrics=metrics)

    def _backward_native(self, x: Tensor, ids: Tensor, weights: Tensor, scores: Tensor, d_update: Tensor,
                         d_aux: Tensor | None, d_scores: Tensor | None,
                         expert_wgrad: str = "native",
                         saved: tuple | None = None,
                         forward_ws: tuple[Tensor, Tensor] | None = None) -> dict[str, Tensor]:
        """Gradients of x and of every parameter (``spx_layer_backward`` for the
        routed experts -- their weight gradients included, on tcgen05 grouped
        GEMMs -- and the router scores; library GEMMs for the router's weight
        gradient and the shared SwiGLU).  The GEMM1 (forward or recomputed) and
        the dh' GEMM write the x rows and the dU rows they gather in dispatch
        order on the side, and the weight-gradient GEMMs read those (the down
        projection's with the routing weights on its hidden rows);
        ``expert_wgrad="native_gathered"`` skips the two P x d copies (less
        memory, slower: the weight-gradient kernels then gather the rows
        themselves), and ``expert_wgrad="library"`` computes the experts' weight
        gradients with ``torch._grouped_mm`` from the sorted rows instead (a
        comparison seam for the tests).  ``saved``: the activations the
        forward wrote for this backward (``_training_saves``); GEMM1 is then
        not recomputed.  ``forward_ws``: (workspace, expert utilization) of that
        forward when no forward of this layer ran since; its dispatch is read
        from there instead of being recomputed."""

        import torch.nn.functional as F

        config = self.config
        device = x.device
        T, d = x.shape
        k = ids.shape[-1]
        E, I = config.num_experts, config.resolved_inter_dim
        P = T * k
        kI = -(-I // 64) * 64
        lib = _lib.load()
        dims = layer_dims(config, T, k)
        packed = self._packed(device, T, k)
        nbytes = _lib.ctypes.c_size_t()
        _lib.check(lib.spx_layer_backward_sizes(dims, nbytes), "spx_layer_backward_sizes")
        ws = torch.empty(nbytes.value, dtype=torch.uint8, device=device)
        d_hidden = torch.empty(T, d, dtype=torch.bfloat16, device=device)
        d_logits = torch.empty(T, E, dtype=torch.bfloat16, device=device)
        h_sorted = torch.empty(P, I, dtype=torch.bfloat16, device=device)
        dgu = torch.empty(P, 2 * kI, dtype=torch.bfloat16, device=device)
        counts = torch.empty(E, dtype=torch.int32, device=device)
        # the experts' weight gradients come out of the same native call (tcgen05 grouped GEMMs over
        # the sorted rows) when the hidden width allows 16-byte rows
        native_wgrad = I % 8 == 0 and expert_wgrad in ("native", "native_gathered")
        copies = not (native_wgrad and expert_wgrad == "native_gathered")
        if not copies:
            saved = None
        if saved is not None:
            x_sorted = saved[0]
        else:
            x_sorted = torch.empty(P, d, dtype=torch.bfloat16, device=device) if copies else None
        du_sorted = torch.empty(P, d, dtype=torch.bfloat16, device=device) if copies else None
        wgrads = {n: torch.empty(E, *shape, dtype=torch.bfloat16, device=device) if native_wgrad else None
                  for n, shape in (("gate", (d, I)), ("up", (d, I)), ("down", (I, d)))}
        residency = self.residency
        mask = None if residency.is_full else residency.resident_mask.to(device=device).contiguous()
        lut = softplus_table(device) if config.router_score_transform == "softplus" else None
        pw = _lib.PackedWeights(
            router_weight=_lib.ptr(packed["router_weight"]),
            router_bias=_lib.ptr(packed["router_bias"]),
            expert_w1=_lib.ptr(packed["expert_w1"]),
            expert_w2=_lib.ptr(packed["expert_w2"]),
            shared_w1=_lib.ptr(packed["shared_w1"]),
            shared_w2=_lib.ptr(packed["shared_w2"]),
            softplus_table=_lib.ptr(lut),
            resident_mask=_lib.ptr(mask),
        )
        gate = self.experts.gate_proj.detach().contiguous()
        up = self.experts.up_proj.detach().contiguous()
        down = self.experts.down_proj.detach().contiguous()
        du = d_update.reshape(T, d).to(torch.bfloat16).contiguous()
        dsc = None if d_scores is None else d_scores.reshape(T, E).to(torch.bfloat16).contiguous()
        dax = None if d_aux is None else d_aux.reshape(1).to(torch.bfloat16).contiguous()
        gr = _lib.LayerGrads(
            expert_ids=ids.data_ptr(), routing_weights=weights.data_ptr(), router_scores=scores.data_ptr(),
            gate_proj=gate.data_ptr(), up_proj=up.data_ptr(), down_proj=down.data_ptr(),
            d_update=du.data_ptr(), d_scores=_lib.ptr(dsc), d_aux=_lib.ptr(dax),
            d_hidden_experts=d_hidden.data_ptr(), d_logits=d_logits.data_ptr(), x_sorted=_lib.ptr(x_sorted),
            h_sorted=h_sorted.data_ptr(), du_sorted=_lib.ptr(du_sorted), dgu_sorted=dgu.data_ptr(),
            expert_counts=counts.data_ptr(), d_gate_proj=_lib.ptr(wgrads["gate"]),
            d_up_proj=_lib.ptr(wgrads["up"]), d_down_proj=_lib.ptr(wgrads["down"]),
            saved_gu=None if saved is None else saved[1].data_ptr(),
            router_logits=None if saved is None else _lib.ptr(saved[2]),
            forward_workspace=None if forward_ws is None else forward_ws[0].data_ptr(),
            expert_utilization=None if forward_ws is None else forward_ws[1].data_ptr(),
        )
        stream = torch.cuda.current_stream(device).cuda_stream
        _lib.check(lib.spx_layer_backward(dims, pw, x.data_ptr(), gr, ws.data_ptr(), stream), "spx_layer_backward")

        grads: dict[str, Tensor] = {}
        w_router = self.router.proj.weight
        grads["router.proj.weight"] = d_logits.t() @ x
        if self.router.proj.bias is not None:
            grads["router.proj.bias"] = d_logits.float().sum(0).to(torch.bfloat16)
        dx = torch.addmm(d_hidden, d_logits, w_router.detach())  # one rounding: d_hidden + d_logits @ W
        if native_wgrad:
            grads["experts.gate_proj"] = wgrads["gate"]
            grads["experts.up_proj"] = wgrads["up"]
            grads["experts.down_proj"] = wgrads["down"]
        else:
            offs = torch.cumsum(counts, 0, dtype=torch.int32)
            grads["experts.gate_proj"] = _grouped_wgrad(x_sorted, dgu[:, :I], counts, offs)
            grads["experts.up_proj"] = _grouped_wgrad(x_sorted, dgu[:, kI:kI + I], counts, offs)
            grads["experts.down_proj"] = _grouped_wgrad(h_sorted, du_sorted, counts, offs)  # h_sorted: h * w
        if self.shared is not None and _shared_bwd_native(self.shared, x):
            # Shared SwiGLU backward without autograd: [gate | up] in one GEMM,
            # the elementwise part in one kernel (spx_swiglu_backward_rows,
            # unit weights), [d gate | d up] against [W_g | W_u] in one GEMM
            # each for the input and the weight gradients.
            sh = self.shared
            wg, wu, wd = (w.detach() for w in (sh.gate_projection.weight, sh.up_projection.weight,
                                               sh.down_projection.weight))
            S = wg.shape[0]
            T = x.shape[0]
            w1 = torch.cat([wg, wu], 0)
            if saved is not None and saved[3] is not None:
                # the forward's own gate | up values (chunk layout: per chunk, gate then up)
                gate_up, chunk = saved[3]
            else:
                gate_up, chunk = F.linear(x, w1), S
            d_h = du.mm(wd)
            h_s = torch.empty(T, S, dtype=torch.bfloat16, device=device)
            dgu_s = torch.empty(T, 2 * S, dtype=torch.bfloat16, device=device)
            ones = torch.ones(T, dtype=torch.bfloat16, device=device)
            order = torch.arange(T, dtype=torch.int32, device=device)
            d_w = torch.empty(T, dtype=torch.float32, device=device)
            _lib.check(lib.spx_swiglu_backward_rows(gate_up.data_ptr(), gate_up.shape[1], chunk, d_h.data_ptr(), S,
                                                    ones.data_ptr(), order.data_ptr(), T, S, S, h_s.data_ptr(),
                                                    dgu_s.data_ptr(), d_w.data_ptr(), stream),
                       "spx_swiglu_backward_rows")
            dx = torch.addmm(dx, dgu_s, w1)  # one rounding: dx + [d gate | d up] @ [W_g | W_u]
            dw1 = dgu_s.t().mm(x)
            grads["shared.gate_projection.weight"] = dw1[:S]
            grads["shared.up_projection.weight"] = dw1[S:]
            grads["shared.down_projection.weight"] = du.t().mm(h_s)
        elif self.shared is not None:
            sh = self.shared
            ws_ = [sh.gate_projection.weight, sh.up_projection.weight, sh.down_projection.weight]
            with torch.enable_grad():
                xs = x.detach().requires_grad_(True)
                leaves = [w.detach().requires_grad_(True) for w in ws_]
                out = F.linear(F.silu(F.linear(xs, leaves[0])) * F.linear(xs, leaves[1]), leaves[2])
                g = torch.autograd.grad(out, [xs] + leaves, du)
            dx = dx + g[0]
            grads["shared.gate_projection.weight"] = g[1]
            grads["shared.up_projection.weight"] = g[2]
            grads["shared.down_projection.weight"] = g[3]
        grads["x"] = dx
        return grads


def _shared_bwd_native(shared, x: Tensor) -> bool:
    """Whether the shared SwiGLU backward fits spx_swiglu_backward_rows (no biases, rows in 16-byte units)."""

    layers = (shared.gate_projection, shared.up_projection, shared.down_projection)
    S = shared.gate_projection.weight.shape[0]
    return (all(getattr(m, "bias", None) is None for m in layers) and S % 8 == 0 and x.dim() == 2
            and x.dtype == torch.bfloat16)


def _grouped_wgrad(a_sorted: Tensor, b_sorted: Tensor, counts: Tensor, offs: Tensor) -> Tensor:
    """Per expert ``a_e^T @ b_e`` over the expert's sorted rows ([E, a_cols, b_cols], BF16).

    One grouped library GEMM (``torch._grouped_mm``, groups along K) when the
    installed PyTorch provides it for this device, else one GEMM per expert.
    """

    E = counts.numel()
    if hasattr(torch, "_grouped_mm"):
        try:
            return torch._grouped_mm(a_sorted.t(), b_sorted, offs=offs)
        except (RuntimeError, TypeError, NotImplementedError):
            if not b_sorted.is_contiguous():  # a column slice: the grouped GEMM may want it dense
                try:
                    return torch._grouped_mm(a_sorted.t(), b_sorted.contiguous(), offs=offs)
                except (RuntimeError, TypeError, NotImplementedError):
                    pass
    out = torch.zeros(E, a_sorted.shape[1], b_sorted.shape[1], dtype=a_sorted.dtype, device=a_sorted.device)
    ends = offs.tolist()
    start = 0
    for e, end in enumerate(ends):
        if end > start:
            out[e] = a_sorted[start:end].t() @ b_sorted[start:end]
        start = end
    return out


class _LayerFunction(torch.autograd.Function):
    """Autograd node of one layer: native forward, native backward."""

    @staticmethod
    def forward(ctx, mixer, holder, names, hidden_states, *params):
        saved = mixer._training_saves(hidden_states)
        out = mixer._forward_native(hidden_states, None, saved=saved)
        ctx.saved_activations = saved
        # the forward's dispatch stays in the layer's workspace until its next forward
        ctx.forward_ws = (*mixer._last_forward, out.metrics["expert_utilization"]) if saved is not None else None
        # outputs without a gradient (usually the router scores) reach backward
        # as None rather than as materialised zeros
        ctx.set_materialize_grads(False)
        m = out.metrics
        holder["metrics"] = m
        ctx.mixer = mixer
        ctx.names = names
        ctx.shape = hidden_states.shape
        x = hidden_states.reshape(-1, hidden_states.shape[-1]).contiguous()
        k = m["expert_ids"].shape[-1]
        ctx.save_for_backward(x, m["expert_ids"].reshape(-1, k), m["routing_weights"].reshape(-1, k),
                              m["router_scores"].reshape(x.shape[0], -1))
        ctx.mark_non_differentiable(m["expert_ids"], m["routing_weights"])
        return out.update, out.auxiliary_loss, m["router_scores"]

    @staticmethod
    def backward(ctx, d_update, d_aux, d_scores):
        x, ids, weights, scores = ctx.saved_tensors
        if d_update is None:
            d_update = torch.zeros(ctx.shape, dtype=torch.bfloat16, device=x.device)
        forward_ws = None
        if ctx.forward_ws is not None and ctx.forward_ws[0] == ctx.mixer._ws_generation:
            forward_ws = ctx.forward_ws[1:]  # no forward of this layer since: its dispatch is still there
        grads = ctx.mixer._backward_native(x, ids, weights, scores, d_update, d_aux, d_scores,
                                           saved=ctx.saved_activations, forward_ws=forward_ws)
        ctx.saved_activations = None
        ctx.forward_ws = None
        return (None, None, None, grads["x"].reshape(ctx.shape), *[grads[n] for n in ctx.names])


class RMSNorm(nn.Module):
    """RMS normalization with float32 variance accumulation (nn/norm.py:9-31)."""

    def __init__(self, d_model: int, eps: float = 1e-6, *, device=None, dtype=None) -> None:
        super().__init__()
        if d_model <= 0:
            raise ValueError("d_model must be positive")
        if eps <= 0:
            raise ValueError("eps must be positive")
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d_model, device=device, dtype=dtype))

    def forward(self, hidden_states: Tensor) -> Tensor:
        variance = hidden_states.float().square().mean(dim=-1, keepdim=True)
        normalized = hidden_states * torch.rsqrt(variance + self.eps).to(hidden_states.dtype)
        return normalized * self.weight.to(hidden_states.dtype)


class B200ChannelBlock(nn.Module):
    """The channel half of ``SPALMERBlock.forward`` (modeling.py:283-302):
    ``h + channel_mixer(channel_norm(h)).update``, fused into one native call
    (``spx_block_channel_forward``: the RMSNorm feeds every GEMM, the residual
    add runs in the combine).  ``forward`` returns ``(h_out, mixer_output)``;
    ``mixer_output.update`` is the layer update itself.  Forward only: under
    autograd it runs the unfused modules (norm, mixer with its backward, add).
    """

    def __init__(self, config, *, channel_norm: RMSNorm | None = None,
                 channel_mixer: "B200MicroExpertChannelMixer | None" = None, eps: float = 1e-6) -> None:
        super().__init__()
        config = coerce_config(config)
        self.channel_mixer = channel_mixer if channel_mixer is not None else B200MicroExpertChannelMixer(config)
        self.channel_norm = channel_norm if channel_norm is not None else RMSNorm(config.d_model, eps)

    def forward(self, hidden_states: Tensor) -> tuple[Tensor, ChannelMixerOutput]:
        mixer = self.channel_mixer
        if mixer.experts.expert_offload_enabled or (torch.is_grad_enabled() and (
            hidden_states.requires_grad or any(p.requires_grad for p in self.parameters())
        )):
            out = mixer(self.channel_norm(hidden_states))
            return hidden_states + out.update, out
        if hidden_states.ndim != 3 or hidden_states.shape[-1] != mixer.config.d_model:
            raise ValueError(f"hidden_states must be [batch, seq, {mixer.config.d_model}]")
        if not hidden_states.is_cuda:
            raise RuntimeError("the B200 micro-expert layer requires CUDA hidden states")
        weight = self.channel_norm.weight.detach().to(torch.bfloat16).contiguous()
        hidden_out = torch.empty_like(hidden_states, dtype=torch.bfloat16)
        out = mixer._forward_native(hidden_states, None, block=(weight, float(self.channel_norm.eps), hidden_out))
        return hidden_out, out


MicroExpertChannelMixer = B200MicroExpertChannelMixer


def route(logits: Tensor, top_k: int, *, transform: str = "softplus",
          resident_mask: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:
    """Scores, top-k ids and weights from BF16 logits ``[T, E]`` (spx_route).

    Restates ``SurpriseRouter`` score transform + ``select_least_surprised_experts``
    (experts/router.py:52-95) given logits.
    """

    if logits.ndim != 2 or logits.dtype != torch.bfloat16 or not logits.is_cuda:
        raise ValueError("logits must be a [T, E] bfloat16 CUDA tensor")
    T, E = logits.shape
    lib = _lib.load()
    device = logits.device
    dims = _lib.LayerDims(tokens=T, d_model=64, num_experts=E, inter_dim=16, shared_dim=0, top_k=top_k,
                          score_transform=0 if transform == "softplus" else 1, execution_loop=0)
    nbytes = _lib.ctypes.c_size_t()
    _lib.check(lib.spx_layer_sizes(dims, nbytes, None), "spx_layer_sizes")
    ws = torch.zeros(nbytes.value, dtype=torch.uint8, device=device)
    scores = torch.empty(T, E, dtype=torch.bfloat16, device=device)
    ids = torch.empty(T, top_k, dtype=torch.long, device=device)
    weights = torch.empty(T, top_k, dtype=torch.bfloat16, device=device)
    lut = softplus_table(device) if transform == "softplus" else None
    mask = None if resident_mask is None else resident_mask.to(device=device, dtype=torch.bool).contiguous()
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.check(
        lib.spx_route(dims, logits.contiguous().data_ptr(), _lib.ptr(lut), _lib.ptr(mask), scores.data_ptr(),
                      ids.data_ptr(), weights.data_ptr(), ws.data_ptr(), stream),
        "spx_route",
    )
    return scores, ids, weights


def rms_norm(hidden: Tensor, weight: Tensor, eps: float = 1e-6) -> Tensor:
    """``RMSNorm.forward`` (nn/norm.py:28-31) of BF16 rows on the device
    (spx_rmsnorm_rows): the pass ``B200ChannelBlock`` fuses before the layer.
    ``hidden`` [..., d] BF16 CUDA, ``weight`` [d]; returns BF16 rows [..., d]."""

    if hidden.dtype != torch.bfloat16 or not hidden.is_cuda:
        raise ValueError("hidden must be a bfloat16 CUDA tensor")
    d = hidden.shape[-1]
    if weight.shape != (d,):
        raise ValueError(f"weight must be [{d}]")
    rows = hidden.contiguous().view(-1, d)
    w = weight.detach().to(device=hidden.device, dtype=torch.bfloat16).contiguous()
    out = torch.empty_like(rows)
    lib = _lib.load()
    stream = torch.cuda.current_stream(hidden.device).cuda_stream
    _lib.check(lib.spx_rmsnorm_rows(rows.data_ptr(), w.data_ptr(), float(eps), rows.shape[0], d, out.data_ptr(), d,
                                    stream), "spx_rmsnorm_rows")
    return out.view(hidden.shape)


def dispatch(expert_ids: Tensor, num_experts: int) -> tuple[Tensor, Tensor]:
    """Stable permutation of pairs by expert and per-expert counts (spx_dispatch).

    Restates ``argsort(expert_index, stable=True)`` and ``_pair_counts``
    (experts/bank.py:721-723, 981-985).
    """

    if expert_ids.ndim != 2 or expert_ids.dtype != torch.long or not expert_ids.is_cuda:
        raise ValueError("expert_ids must be a [T, k] int64 CUDA tensor")
    T, k = expert_ids.shape
    lib = _lib.load()
    device = expert_ids.device
    dims = _lib.LayerDims(tokens=T, d_model=64, num_experts=num_experts, inter_dim=16, shared_dim=0,
                          top_k=k, score_transform=1, execution_loop=0)
    nbytes = _lib.ctypes.c_size_t()
    _lib.check(lib.spx_layer_sizes(dims, nbytes, None), "spx_layer_sizes")
    ws = torch.zeros(nbytes.value, dtype=torch.uint8, device=device)
    order = torch.empty(T * k, dtype=torch.int32, device=device)
    counts = torch.empty(num_experts, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    _lib.check(
        lib.spx_dispatch(dims, expert_ids.contiguous().data_ptr(), order.data_ptr(), counts.data_ptr(),
                         ws.data_ptr(), stream),
        "spx_dispatch",
    )
    return order, counts


__all__ = [
    "B200ChannelBlock",
    "B200MicroExpertChannelMixer",
    "RMSNorm",
    "ChannelMixerOutput",
    "ExpertPotentiationController",
    "ExpertResidency",
    "MicroExpertBank",
    "MicroExpertChannelMixer",
    "MicroExpertsConfig",
    "NativeExpertPrecisionError",
    "SurpriseRouter",
    "SwiGLU",
    "dispatch",
    "rms_norm",
    "route",
    "softplus_table",
]
