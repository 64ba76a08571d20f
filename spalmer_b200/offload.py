"""Paged expert offload for the B200 layer.

The reference (mESmaC/spalmer ``src/spalmer/experts/offload.py`` and
``experts/bank.py:95-407, 781-899``) keeps each layer's complete expert bank
on the CPU and stages the experts a forward selects into a bounded device
cache of ``capacity`` experts; routing stays unrestricted and the selected
experts execute page by page, each page no larger than the cache.

Here the same policy drives a device cache held in the kernels' packed
layout:

* the CPU masters (the module's own parameters, optionally page-locked) are
  packed once into pinned host buffers in the layout ``spx_pack_weights``
  writes, so staging an expert is one host-to-device copy per packed array
  (runs of consecutive experts and slots merge into one copy);
* ``spx_layer_paged_begin`` routes and dispatches; the host reads the
  per-expert pair counts (the one synchronisation, as in the reference),
  plans the pages, and for each page copies the missing experts into their
  slots on a copy stream and runs ``spx_layer_paged_experts`` on the page
  (split into chunks so a chunk's GEMMs overlap the next chunk's copies);
* ``spx_layer_paged_finish`` adds the shared SwiGLU and combines.

Pages write the same rows an unpaged pass writes, so the update equals the
unpaged layer's bit for bit.  The cache policy (page plan, retained rows,
least-recently-used spare slots, the four counters) follows the reference
step for step and is checked against traces of the reference itself
(``tests/golden/paging_traces.json``).  Retained experts keep their slot;
the reference re-lays its cache out in id order, which changes no result.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Any
from weakref import ref

import numpy as np
import torch
from torch import Tensor, nn

from spalmer_b200 import _lib


# ---------------------------------------------------------------- host policy
def power_of_two_count_buckets(counts: Sequence[int]) -> tuple[tuple[int, tuple[int, ...]], ...]:
    """Positions of positive counts grouped by next-power-of-two capacity,
    buckets in ascending capacity, positions ascending (bank.py:988-1010)."""

    grouped: dict[int, list[int]] = {}
    for position, raw in enumerate(counts):
        count = int(raw)
        if count < 1:
            raise ValueError("count buckets require positive group counts")
        grouped.setdefault(1 << (count - 1).bit_length(), []).append(position)
    return tuple((cap, tuple(pos)) for cap, pos in sorted(grouped.items()))


def page_plan(counts: Sequence[int] | np.ndarray, capacity: int, *, loop: bool = False) -> list[tuple[int, ...]]:
    """The execution pages of one forward from the per-expert pair counts.

    Grouped execution (bank.py:821-866): the selected experts (count > 0) in
    id order, grouped into power-of-two count buckets, each bucket cut into
    runs of ``capacity``.  Loop execution (bank.py:781-818): the sorted
    selected ids cut into runs of ``capacity``.
    """

    if capacity < 1:
        raise ValueError("cache capacity must be positive")
    counts = np.asarray(counts).reshape(-1)
    selected = [int(e) for e in np.flatnonzero(counts > 0)]
    if loop:
        return [tuple(selected[i:i + capacity]) for i in range(0, len(selected), capacity)]
    pages: list[tuple[int, ...]] = []
    for _, positions in power_of_two_count_buckets([int(counts[e]) for e in selected]):
        for offset in range(0, len(positions), capacity):
            pages.append(tuple(selected[p] for p in positions[offset:offset + capacity]))
    return pages


@dataclass(frozen=True)
class StagePlan:
    """One cache update: the new id set, copies to make, and its counter delta."""

    expert_ids: tuple[int, ...]
    slots: dict[int, int]                 # expert -> slot after the update
    incoming: tuple[tuple[int, int], ...]  # (expert, slot) to copy, ascending expert
    evicted: tuple[int, ...]
    lru: tuple[int, ...]


class ExpertCachePolicy:
    """Host state of one layer's expert cache (bank.py:241-365): the staged
    ids, the slot of each, the least-recently-used order and the counters
    (stage operations, transferred rows, evicted rows, transferred bytes)."""

    def __init__(self, num_experts: int, capacity: int, bytes_per_row: int) -> None:
        if not 1 <= capacity <= num_experts:
            raise ValueError(f"expert cache capacity must lie in [1, {num_experts}]; got {capacity}")
        self.num_experts = num_experts
        self.capacity = capacity
        self.bytes_per_row = bytes_per_row
        self.cached_ids: tuple[int, ...] = ()
        self.slots: dict[int, int] = {}
        self.lru: list[int] = []
        self.counters = [0, 0, 0, 0]

    def plan_rows(self, expert_ids: Sequence[int], *, force: bool = False) -> StagePlan | None:
        """Stage exactly ``expert_ids`` (sorted, unique); None when nothing
        changes (``_stage_expert_rows`` returns early then)."""

        ids = tuple(int(e) for e in expert_ids)
        if not ids:
            raise ValueError("at least one expert must be staged")
        if len(ids) > self.capacity:
            raise ValueError(f"{len(ids)} resident experts exceed cache capacity {self.capacity}")
        if tuple(sorted(set(ids))) != ids:
            raise ValueError("staged expert ids must be unique and sorted")
        if ids[0] < 0 or ids[-1] >= self.num_experts:
            raise ValueError(f"expert ids must lie in [0, {self.num_experts})")
        if not force and ids == self.cached_ids:
            return None
        retained = () if force else tuple(e for e in ids if e in self.slots)
        keep = set(retained)
        incoming = tuple(e for e in ids if e not in keep)
        wanted = set(ids)
        evicted = tuple(e for e in self.cached_ids if e not in wanted)
        slots = {e: self.slots[e] for e in retained}
        taken = set(slots.values())
        free = [s for s in range(self.capacity) if s not in taken]
        for e, s in zip(incoming, free):
            slots[e] = s
        return StagePlan(ids, slots, tuple((e, slots[e]) for e in incoming), evicted, ids)

    def plan_page(self, required_ids: Sequence[int]) -> tuple[StagePlan | None, tuple[int, ...]]:
        """``_stage_execution_page``: the required ids plus the most recently
        used others in spare slots; returns the stage plan (or None) and the
        LRU order after the page."""

        required = tuple(sorted({int(e) for e in required_ids}))
        if not required:
            raise ValueError("an execution page needs at least one expert")
        if len(required) > self.capacity:
            raise ValueError(f"{len(required)} requested experts exceed cache capacity {self.capacity}")
        keep = set(required)
        for e in reversed(self.lru):
            if len(keep) >= self.capacity:
                break
            keep.add(e)
        plan = self.plan_rows(tuple(sorted(keep)))
        lru = tuple(e for e in self.lru if e in keep and e not in required) + required
        return plan, lru

    def commit(self, plan: StagePlan | None, lru: Sequence[int] | None = None) -> None:
        if plan is not None:
            self.cached_ids = plan.expert_ids
            self.slots = dict(plan.slots)
            self.lru = list(plan.lru)
            self.counters[0] += 1
            self.counters[1] += len(plan.incoming)
            self.counters[2] += len(plan.evicted)
            self.counters[3] += len(plan.incoming) * self.bytes_per_row
        if lru is not None:
            self.lru = list(lru)


# ---------------------------------------------------------------- device cache
_PACKED_ARRAYS = ("expert_w1", "expert_w2")
_PACKED_ARRAYS_MX = ("expert_w1_mx", "expert_w1_mx_scales", "expert_w2_mx", "expert_w2_mx_scales")


class PagedExpertCache:
    """One layer's expert cache: pinned packed masters on the host, ``capacity``
    packed slots on the device, the policy, and the copy stream."""

    def __init__(self, bank: nn.Module, target: torch.device, capacity: int, *, non_blocking: bool,
                 paging: bool, copy_chunk: int = 32) -> None:
        config = bank.config
        self.config = config
        self.target = target
        self.capacity = capacity
        self.non_blocking = non_blocking
        self.paging = paging
        self.copy_chunk = max(1, int(copy_chunk))
        bytes_per_row = bank.parameters_per_expert * bank.gate_proj.element_size()
        self.policy = ExpertCachePolicy(config.num_experts, capacity, bytes_per_row)
        self._bank_ref = ref(bank)
        self.host: dict[str, Tensor] = {}     # [E, bytes per expert] pinned
        self.device: dict[str, Tensor] = {}   # [capacity, bytes per expert]
        self.quant_error: Tensor | None = None  # [E] low-precision reconstruction error (device), see _pack_host
        self._master_key: tuple | None = None
        self.copy_stream: torch.cuda.Stream | None = None
        self.physical_bytes_copied = 0  # packed bytes moved host -> device (all arrays, padding included)
        self.last_chunks = 0
        # CTAs of the staging copy; while one runs beside a chunk's GEMMs,
        # those GEMMs leave this many SMs free for it.
        self.stage_ctas = 16

    # -- packing
    def _bank(self) -> nn.Module:
        bank = self._bank_ref()
        if bank is None:
            raise RuntimeError("the expert bank owning this cache no longer exists")
        return bank

    def _master_tensors(self) -> tuple[Tensor, Tensor, Tensor]:
        bank = self._bank()
        return bank.gate_proj, bank.up_proj, bank.down_proj

    def masters_key(self) -> tuple:
        return tuple((t.data_ptr(), t._version, t.dtype, t.device) for t in self._master_tensors())

    def ensure_packed(self) -> bool:
        """(Re)pack the CPU masters into the pinned host buffers when they
        changed; returns True when it packed."""

        key = self.masters_key()
        if key == self._master_key and self.host:
            return False
        self._pack_host()
        self._master_key = key
        return True

    def _pack_dims(self, experts: int) -> _lib.LayerDims:
        from spalmer_b200.experts import layer_dims

        dims = layer_dims(self.config, 1024, 1)
        dims.num_experts = experts
        dims.shared_dim = 0
        return dims

    def per_expert_bytes(self) -> dict[str, int]:
        lib = _lib.load()
        sizes = _lib.PackedSizes()
        _lib.check(lib.spx_layer_sizes(self._pack_dims(1), None, sizes), "spx_layer_sizes")
        out = {"expert_w1": 2 * sizes.expert_w1, "expert_w2": 2 * sizes.expert_w2}
        lane = self._pack_dims(1).mxfp8_lane
        if lane:
            for name in _PACKED_ARRAYS_MX:
                out[name] = getattr(sizes, name)
        if lane == 2:
            out["expert_nvfp4_amax"] = sizes.expert_nvfp4_amax
        return out

    def _pack_host(self) -> None:
        if self.target.type != "cuda":
            raise RuntimeError("the paged B200 layer packs and executes experts on a CUDA device")
        lib = _lib.load()
        gate, up, down = self._master_tensors()
        E = self.config.num_experts
        per = self.per_expert_bytes()
        pin = gate.device.type == "cpu"
        host = {name: torch.empty(E, n, dtype=torch.uint8, pin_memory=pin) for name, n in per.items()}
        dev = self.target
        # reconstruction error of every expert's low-precision copies (bank.py:526-592), from
        # the same device copies of the masters
        from spalmer_b200.experts import _QUANT_ERROR_FORMATS

        qfmt = _QUANT_ERROR_FORMATS.get(self.config.expert_weight_format)
        quant_error = torch.zeros(E, dtype=torch.float32, device=dev) if qfmt is not None else None
        stream = torch.cuda.current_stream(dev)
        step = 32
        with torch.cuda.device(dev):
            for e0 in range(0, E, step):
                n = min(step, E - e0)
                dims = self._pack_dims(n)
                g = gate.detach()[e0:e0 + n].to(dev, torch.bfloat16).contiguous()
                u = up.detach()[e0:e0 + n].to(dev, torch.bfloat16).contiguous()
                dn = down.detach()[e0:e0 + n].to(dev, torch.bfloat16).contiguous()
                router = torch.zeros(n, self.config.d_model, dtype=torch.bfloat16, device=dev)
                sizes = _lib.PackedSizes()
                _lib.check(lib.spx_layer_sizes(dims, None, sizes), "spx_layer_sizes")
                scratch = torch.empty(max(1, sizes.router_weight), dtype=torch.int16, device=dev)
                out = {name: torch.empty(n, nb, dtype=torch.uint8, device=dev) for name, nb in per.items()}
                src = _lib.ReferenceWeights(router_weight=router.data_ptr(), gate_proj=g.data_ptr(),
                                            up_proj=u.data_ptr(), down_proj=dn.data_ptr())
                _lib.check(lib.spx_pack_weights(dims, src, scratch.data_ptr(), out["expert_w1"].data_ptr(),
                                                out["expert_w2"].data_ptr(), None, None, stream.cuda_stream),
                           "spx_pack_weights (expert masters)")
                if qfmt is not None:
                    _lib.check(lib.spx_expert_quant_error(dims, src, qfmt, quant_error[e0:].data_ptr(),
                                                          stream.cuda_stream), "spx_expert_quant_error")
                if dims.mxfp8_lane:
                    from spalmer_b200.experts import pack_lowp_experts

                    lowp = pack_lowp_experts(dims, src, sizes, lambda nb: torch.empty(nb, dtype=torch.uint8, device=dev),
                                             stream.cuda_stream)
                    for name in out:
                        if name in lowp:
                            out[name].copy_(lowp[name][:out[name].numel()].view(n, -1))
                for name, t in out.items():
                    host[name][e0:e0 + n].copy_(t)
        stream.synchronize()
        self.host = host
        self.quant_error = quant_error
        if not self.device:
            self.device = {name: torch.empty(self.capacity, n, dtype=torch.uint8, device=dev)
                           for name, n in per.items()}

    # -- copies
    def _stage_copies(self, pairs: Tensor, n: int, stream: torch.cuda.Stream) -> None:
        """Copy ``n`` whole experts from the pinned host bank into their slots:
        ``pairs`` is a device int32 tensor [n, 2] of (expert, slot).  One
        ``spx_stage_expert_slots`` launch; the GPU reads the host memory."""

        if n == 0:
            return
        lib = _lib.load()
        names = list(self.device)
        k = len(names)
        src = (_lib.ctypes.c_void_p * k)(*(self.host[nm].data_ptr() for nm in names))
        dst = (_lib.ctypes.c_void_p * k)(*(self.device[nm].data_ptr() for nm in names))
        nbytes = (_lib.ctypes.c_int64 * k)(*(self.device[nm].shape[1] for nm in names))
        _lib.check(lib.spx_stage_expert_slots(src, dst, nbytes, k, pairs.data_ptr(), n, self.config.num_experts,
                                              self.capacity, self.stage_ctas, stream.cuda_stream),
                   "spx_stage_expert_slots")
        self.physical_bytes_copied += n * sum(nbytes)

    def stage_now(self, plan: StagePlan | None, lru: Sequence[int] | None = None) -> None:
        """Apply a plan on the current stream (no overlap; used outside a forward)."""

        if plan is not None and plan.incoming:
            self.ensure_packed()
            stream = torch.cuda.current_stream(self.target)
            pairs = torch.tensor(plan.incoming, dtype=torch.int32).pin_memory().to(self.target, non_blocking=True)
            self._stage_copies(pairs, len(plan.incoming), stream)
        self.policy.commit(plan, lru)

    def packed_weights(self, lanes: Tensor | None) -> _lib.PackedWeights:
        d = self.device
        return _lib.PackedWeights(
            expert_w1=d["expert_w1"].data_ptr(), expert_w2=d["expert_w2"].data_ptr(),
            expert_lane_mxfp8=_lib.ptr(lanes),
            expert_w1_mx=_lib.ptr(d.get("expert_w1_mx")), expert_w1_mx_scales=_lib.ptr(d.get("expert_w1_mx_scales")),
            expert_w2_mx=_lib.ptr(d.get("expert_w2_mx")), expert_w2_mx_scales=_lib.ptr(d.get("expert_w2_mx_scales")),
            expert_nvfp4_amax=_lib.ptr(d.get("expert_nvfp4_amax")),
        )

    @property
    def cache_bytes(self) -> int:
        return sum(t.numel() for t in self.device.values())

    # -- one forward's expert stage
    def run_pages(self, counts: np.ndarray, run_chunk) -> list[tuple[int, ...]]:
        """Stage and execute every page of one forward.  ``run_chunk(page_slot,
        sm_limit)`` launches the expert GEMMs of one chunk on the compute
        stream: ``page_slot`` an int32 device tensor [E] (slot, or -1 outside
        the chunk), ``sm_limit`` the SMs its GEMMs may take (0 = all; set while
        a later chunk's copy runs beside them).  Returns the pages in execution
        order."""

        restaged = None
        if self.ensure_packed() and self.policy.cached_ids:
            # masters changed under a populated cache (load_state_dict): restage it
            self.stage_now(self.policy.plan_rows(self.policy.cached_ids, force=True))
            restaged = torch.cuda.Event()
            restaged.record(torch.cuda.current_stream(self.target))
        E = self.config.num_experts
        loop = self.config.expert_execution == "loop"
        pages = page_plan(counts, self.capacity, loop=loop) if self.paging else []
        if not self.paging:
            selected = tuple(int(e) for e in np.flatnonzero(np.asarray(counts) > 0))
            missing = [e for e in selected if e not in self.policy.slots]
            if missing:
                raise RuntimeError(f"experts {missing} are not resident in the device cache")
            if selected:
                pages = [selected]
        if not pages:
            return []
        if not hasattr(self, "sm_count"):
            self.sm_count = torch.cuda.get_device_properties(self.target).multi_processor_count
        compute = torch.cuda.current_stream(self.target)
        if self.copy_stream is None:
            self.copy_stream = torch.cuda.Stream(self.target)
        copy = self.copy_stream
        # (page, copies (expert, slot), slots, experts) per chunk
        chunks: list[tuple[int, tuple[tuple[int, int], ...], list[int], list[int]]] = []
        for p, page in enumerate(pages):
            if self.paging:
                plan, lru = self.policy.plan_page(page)
                slots = plan.slots if plan is not None else self.policy.slots
                copies = {e: s for e, s in (plan.incoming if plan is not None else ())}
                self.policy.commit(plan, lru)
            else:
                slots, copies = self.policy.slots, {}
            for c0 in range(0, len(page), self.copy_chunk):
                part = list(page[c0:c0 + self.copy_chunk])
                chunks.append((p, tuple((e, slots[e]) for e in part if e in copies), [slots[e] for e in part], part))
        self.last_chunks = len(chunks)
        # One upload per forward: every chunk's slot table [E] and copy pairs.
        n_pairs = sum(len(c[1]) for c in chunks)
        meta = np.full(len(chunks) * E + 2 * n_pairs, -1, dtype=np.int32)
        table = meta[:len(chunks) * E].reshape(len(chunks), E)
        pair_at = []
        off = len(chunks) * E
        for i, (_, copies, slot_list, part) in enumerate(chunks):
            table[i, part] = slot_list
            pair_at.append(off)
            for e, sl in copies:
                meta[off], meta[off + 1] = e, sl
                off += 2
        # The upload goes on the copy stream: the first page's copies need not
        # wait for the compute stream (every earlier forward's GEMMs finished
        # before the host read this forward's counts), so they overlap shared GEMM1.
        with torch.cuda.stream(copy):
            meta_dev = torch.from_numpy(meta).pin_memory().to(self.target, non_blocking=True)
            uploaded = torch.cuda.Event()
            uploaded.record(copy)
        meta_dev.record_stream(compute)
        compute.wait_event(uploaded)
        page_done = restaged  # the restage copies ran on the compute stream
        last_page = -1
        for i, (p, copies, _, part) in enumerate(chunks):
            if p != last_page:
                # slots this page overwrites were last read by the previous page's GEMMs
                if page_done is not None:
                    copy.wait_event(page_done)
                last_page = p
            if copies:
                self._stage_copies(meta_dev[pair_at[i]:pair_at[i] + 2 * len(copies)], len(copies), copy)
                ready = torch.cuda.Event()
                ready.record(copy)
                compute.wait_event(ready)
            copying = any(chunks[j][1] for j in range(i + 1, len(chunks)) if chunks[j][0] == p)
            run_chunk(meta_dev[i * E:(i + 1) * E], self.sm_count - self.stage_ctas if copying else 0)
            if i + 1 == len(chunks) or chunks[i + 1][0] != p:
                page_done = torch.cuda.Event()
                page_done.record(compute)
        compute.wait_stream(copy)
        return pages


# ---------------------------------------------------------------- telemetry / manager
@dataclass(frozen=True, slots=True)
class ExpertOffloadTelemetry:
    """Placement, occupancy and cumulative transfer counters (offload.py:38-100)."""

    enabled: bool
    paging: bool
    target_device: str | None
    capacity: int
    resident_expert_ids: tuple[int, ...]
    layer_count: int
    master_devices: tuple[str, ...]
    master_pinned_by_layer: tuple[bool, ...]
    cache_devices: tuple[str, ...]
    cached_expert_ids_by_layer: tuple[tuple[int, ...], ...]
    master_bytes: int
    cache_bytes: int
    cache_index_bytes: int
    stage_operations: int
    transferred_expert_rows: int
    evicted_expert_rows: int
    transfer_bytes: int

    @property
    def occupancy(self) -> float:
        if not self.capacity:
            return 0.0
        if self.paging:
            occupied = max((len(ids) for ids in self.cached_expert_ids_by_layer), default=0)
        else:
            occupied = len(self.resident_expert_ids)
        return occupied / self.capacity

    @property
    def mode(self) -> str:
        return "paged" if self.paging else "resident"

    @property
    def masters_on_cpu(self) -> bool:
        return bool(self.master_devices) and all(device == "cpu" for device in self.master_devices)

    @property
    def masters_pinned(self) -> bool:
        return bool(self.master_pinned_by_layer) and all(self.master_pinned_by_layer)

    @property
    def caches_on_target(self) -> bool:
        return (self.target_device is not None and bool(self.cache_devices)
                and all(device == self.target_device for device in self.cache_devices))


def _mixers(module: nn.Module) -> tuple[Any, ...]:
    from spalmer_b200.experts import B200MicroExpertChannelMixer

    found = tuple(m for m in module.modules() if isinstance(m, B200MicroExpertChannelMixer))
    if not found:
        raise TypeError("module has no B200 micro-expert layers to offload")
    return found


class ExpertOffloadManager:
    """The caches of every B200 micro-expert layer of one module (offload.py:100-285)."""

    def __init__(self, module: nn.Module, banks: Sequence[nn.Module], target: torch.device, *, capacity: int,
                 non_blocking: bool, paging: bool) -> None:
        self._module_ref = ref(module)
        self._banks = tuple(banks)
        self.target_device = target
        self.capacity = capacity
        self.non_blocking = non_blocking
        self.paging = paging
        self._resident_ids: tuple[int, ...] = ()

    @property
    def resident_ids(self) -> tuple[int, ...]:
        return self._resident_ids

    def stage(self, expert_ids: Sequence[int], *, force: bool = False) -> None:
        """Resident mode: the same sorted id set in every layer (offload.py:152-187)."""

        if self.paging:
            raise RuntimeError("request-global staging is unavailable in paged expert mode")
        raw = tuple(int(e) for e in expert_ids)
        desired = tuple(sorted(set(raw)))
        if len(desired) != len(raw):
            raise ValueError("resident expert ids must be unique")
        if not desired:
            raise ValueError("at least one resident expert id is required")
        if len(desired) > self.capacity:
            raise ValueError(f"{len(desired)} resident experts exceed physical cache capacity {self.capacity}")
        for bank in self._banks:
            bank._stage_expert_rows(desired, force=force)
        self._resident_ids = desired

    def warm(self, expert_ids: Sequence[int]) -> None:
        """Paged mode: seed every layer cache with the same ids (offload.py:189-202)."""

        if not self.paging:
            raise RuntimeError("cache warming is only available in paged expert mode")
        desired = tuple(sorted({int(e) for e in expert_ids}))
        if not desired:
            return
        if len(desired) > self.capacity:
            raise ValueError(f"{len(desired)} warm experts exceed physical cache capacity {self.capacity}")
        for bank in self._banks:
            bank._stage_expert_rows(desired)

    def telemetry(self) -> ExpertOffloadTelemetry:
        counters = [bank.expert_offload_counters for bank in self._banks]
        return ExpertOffloadTelemetry(
            enabled=True, paging=self.paging, target_device=str(self.target_device), capacity=self.capacity,
            resident_expert_ids=self._resident_ids, layer_count=len(self._banks),
            master_devices=tuple(str(b.expert_master_device) for b in self._banks),
            master_pinned_by_layer=tuple(b.expert_masters_pinned for b in self._banks),
            cache_devices=tuple("" if b.expert_cache_device is None else str(b.expert_cache_device)
                                for b in self._banks),
            cached_expert_ids_by_layer=tuple(b.cached_expert_ids for b in self._banks),
            master_bytes=sum(b.expert_master_bytes for b in self._banks),
            cache_bytes=sum(b.expert_cache_bytes for b in self._banks),
            cache_index_bytes=sum(b.expert_cache_index_bytes for b in self._banks),
            stage_operations=sum(c[0] for c in counters),
            transferred_expert_rows=sum(c[1] for c in counters),
            evicted_expert_rows=sum(c[2] for c in counters),
            transfer_bytes=sum(c[3] for c in counters),
        )

    def clear(self) -> None:
        for bank in self._banks:
            bank._clear_expert_offload()
        self._resident_ids = ()


def enable_expert_offload(module: nn.Module, device: torch.device | str, *, cache_size: int | None = None,
                          resident_ids: Sequence[int] | None = None, non_blocking: bool = True,
                          pin_memory: bool | None = None, paging: bool = True) -> ExpertOffloadTelemetry:
    """Place ``module`` on ``device`` with every B200 micro-expert layer's
    expert bank kept on the CPU behind a bounded device cache
    (offload.py:287-397; the module stands where the reference takes its
    model: any module containing ``B200MicroExpertChannelMixer`` layers).

    Paged mode (default): routing stays unrestricted and each forward stages
    the experts it selects; ``resident_ids`` only warms the caches.  Resident
    mode (``paging=False``): ``resident_ids`` (at least ``active_experts``
    ids) become every layer's resident set and routing is restricted to it.
    """

    if module.training:
        raise RuntimeError("expert offload is inference-only; call module.eval() first")
    if getattr(module, "_expert_offload_manager", None) is not None:
        raise RuntimeError("expert offload is already enabled")
    target = torch.device(device)
    if target.type != "cuda":
        raise ValueError("the B200 layer's expert offload needs a CUDA inference device")
    if target.index is None:
        target = torch.device("cuda", torch.cuda.current_device())
    should_pin = True if pin_memory is None else bool(pin_memory)
    mixers = _mixers(module)
    config = mixers[0].config
    residencies = {id(m.residency): m.residency for m in mixers}
    capacity = config.resident_cap if cache_size is None else int(cache_size)
    minimum = 1 if paging else mixers[0].active_experts
    if not minimum <= capacity <= config.num_experts:
        raise ValueError(f"cache_size must lie in [{minimum}, {config.num_experts}]; got {capacity}")
    if paging:
        initial = () if resident_ids is None else tuple(resident_ids)
    elif resident_ids is None:
        initial = tuple(range(max(config.min_resident_experts, mixers[0].active_experts)))
    else:
        initial = tuple(resident_ids)
    initial = tuple(sorted({int(e) for e in initial}))
    if not paging and len(initial) < mixers[0].active_experts:
        raise ValueError(f"the initial cache needs at least active_experts={mixers[0].active_experts} ids")
    if len(initial) > capacity:
        raise ValueError(f"{len(initial)} initial residents exceed physical cache capacity {capacity}")
    banks = tuple(m.experts for m in mixers)
    manager = ExpertOffloadManager(module, banks, target, capacity=capacity, non_blocking=non_blocking,
                                   paging=paging)
    previous = {k: r.ids for k, r in residencies.items()}
    object.__setattr__(module, "_expert_offload_manager", manager)
    try:
        if paging:
            for r in residencies.values():
                r.set(tuple(range(config.num_experts)))
        for bank in banks:
            bank._prepare_expert_offload(target, capacity=capacity, non_blocking=non_blocking,
                                         pin_memory=should_pin, paging=paging)
        module.to(device=target)
        if paging:
            manager.warm(initial)
        else:
            manager.stage(initial)
            for r in residencies.values():
                r.set(initial)
    except BaseException:
        manager.clear()
        object.__setattr__(module, "_expert_offload_manager", None)
        for k, r in residencies.items():
            r.set(previous[k])
        raise
    return manager.telemetry()


def disable_expert_offload(module: nn.Module, *, device: torch.device | str = "cpu") -> None:
    """Drop the caches, restore full residency and place the whole module (offload.py:400-416)."""

    manager = getattr(module, "_expert_offload_manager", None)
    if manager is None:
        return
    manager.clear()
    object.__setattr__(module, "_expert_offload_manager", None)
    for m in _mixers(module):
        m.residency.set(tuple(range(m.config.num_experts)))
    module.to(device=torch.device(device))


def expert_offload_telemetry(module: nn.Module) -> ExpertOffloadTelemetry | None:
    manager = getattr(module, "_expert_offload_manager", None)
    return None if manager is None else manager.telemetry()


__all__ = [
    "ExpertCachePolicy",
    "ExpertOffloadManager",
    "ExpertOffloadTelemetry",
    "PagedExpertCache",
    "StagePlan",
    "disable_expert_offload",
    "enable_expert_offload",
    "expert_offload_telemetry",
    "page_plan",
    "power_of_two_count_buckets",
]
