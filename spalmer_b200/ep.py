"""Expert parallelism for the micro-expert layer: experts sharded over GPUs,
token rows exchanged with NCCL all-to-all.

The reference runs every expert on every rank (its multi-GPU paths are data
parallel); this module adds the expert-parallel layout its survey plans for
the skewed 8-GPU configuration: rank r of G owns experts
[r*E/G, (r+1)*E/G) and its own T_r tokens.  One forward:

1. route (``spx_layer_route``): router GEMM, selection, dispatch of the local
   tokens.  Pairs sorted by expert id are also sorted by owning rank.
2. all-to-all of the per-expert pair counts (E/G int32 per peer), read on the
   host to size the row exchange (the one host synchronisation).
3. ``spx_gather_rows`` packs the hidden-state row of every pair in dispatch
   order; all-to-all-v sends each peer the rows of its experts.
4. ``spx_experts_forward`` runs the received rows through the local experts
   (grouped tcgen05 GEMMs, both precision lanes), unweighted, in receive
   order.
5. all-to-all-v returns the rows; they arrive in the sender's dispatch order.
6. ``spx_combine`` adds bf16(row * routing weight) of each token's k pairs in
   slot order to the shared SwiGLU output (``spx_shared_forward``, computed
   on a side stream while the rows travel).

Every per-row result is computed by the same kernels as the single-GPU layer
on the same operands, so the update is bit-identical to ``spx_layer_forward``
on the same tokens.  The exchange logic (`exchange_plan`, `ExpertParallelMixer`)
is backend-agnostic: `CudaOps` runs libspx; the CPU tests drive the same
exchange with an oracle backend over gloo.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np
import torch
import torch.distributed as dist
from torch import Tensor

from spalmer_b200 import _lib


def experts_per_rank(num_experts: int, world: int) -> int:
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not shard evenly over {world} ranks")
    return num_experts // world


@dataclass
class ExchangePlan:
    """Row counts of one all-to-all round (host integers)."""

    send_rows: list[int]        # rows this rank sends to each peer (its pairs on the peer's experts)
    recv_rows: list[int]        # rows this rank receives from each peer
    recv_expert_counts: np.ndarray  # [G, E_local] rows per (source, local expert), receive order


def exchange_plan(local_counts: np.ndarray, recv_counts: np.ndarray, world: int) -> ExchangePlan:
    """Split sizes from this rank's per-expert pair counts [E] and the counts
    received from every peer for this rank's experts [G * E_local]."""

    local_counts = np.asarray(local_counts, dtype=np.int64).reshape(world, -1)
    recv = np.asarray(recv_counts, dtype=np.int64).reshape(world, -1)
    return ExchangePlan(send_rows=[int(v) for v in local_counts.sum(axis=1)],
                        recv_rows=[int(v) for v in recv.sum(axis=1)],
                        recv_expert_counts=recv)


def receive_expert_ids(plan: ExchangePlan, device: torch.device) -> Tensor:
    """Local expert id of every received row: from each source, its rows for
    local expert 0, then 1, ... (the sender's dispatch order)."""

    counts = torch.from_numpy(plan.recv_expert_counts.reshape(-1)).to(device)
    world, e_local = plan.recv_expert_counts.shape
    ids = torch.arange(e_local, dtype=torch.int64, device=device).repeat(world)
    return torch.repeat_interleave(ids, counts)


class CudaOps:
    """libspx stages for one rank (weights of all experts are kept by the
    module; only this rank's experts are packed)."""

    def __init__(self, mixer: Any, rank: int, world: int, device: torch.device):
        from spalmer_b200.experts import layer_dims, softplus_table

        self.mixer = mixer
        self.config = mixer.config
        self.device = device
        cfg = self.config
        self.E = cfg.num_experts
        self.e_local = experts_per_rank(self.E, world)
        self.e0 = rank * self.e_local
        self.k = mixer.active_experts
        self.d = cfg.d_model
        self._layer_dims = layer_dims
        self.lut = softplus_table(device) if cfg.router_score_transform == "softplus" else None
        self._ws: dict[tuple, Tensor] = {}
        self._router_packs: dict[bool, dict] = {}
        self._expert_packs: dict[bool, dict] = {}

    # ---- packing (kernel layouts depend on the batch class of the call, so
    # router/shared and expert copies are cached per class)
    def _local_dims(self, rows: int) -> _lib.LayerDims:
        dims = self._layer_dims(self.config, max(rows, 1), 1)
        dims.num_experts = self.e_local
        dims.shared_dim = 0
        return dims

    def _pack_router_shared(self, tokens: int) -> dict:
        from spalmer_b200.experts import SMALL_BATCH_TOKENS

        cls = tokens <= SMALL_BATCH_TOKENS
        if cls in self._router_packs:
            return self._router_packs[cls]
        lib = _lib.load()
        m, dev = self.mixer, self.device
        stream = torch.cuda.current_stream(dev).cuda_stream
        full = self._layer_dims(self.config, tokens, self.k)
        sizes = _lib.PackedSizes()
        _lib.check(lib.spx_layer_sizes(full, None, sizes), "spx_layer_sizes")
        s = m.shared
        t = lambda x: None if x is None else x.detach().contiguous()  # noqa: E731
        keep = {
            "router_weight": t(m.router.proj.weight), "router_bias": t(m.router.proj.bias),
            "shared_gate": None if s is None else t(s.gate_projection.weight),
            "shared_up": None if s is None else t(s.up_projection.weight),
            "shared_down": None if s is None else t(s.down_projection.weight),
        }
        empty = lambda n: torch.empty(max(1, n), dtype=torch.int16, device=dev)  # noqa: E731
        pk = {"keep": keep, "router_w": empty(sizes.router_weight),
              "shared_w1": empty(sizes.shared_w1) if sizes.shared_w1 else None,
              "shared_w2": empty(sizes.shared_w2) if sizes.shared_w2 else None}
        src = _lib.ReferenceWeights(router_weight=_lib.ptr(keep["router_weight"]), router_bias=_lib.ptr(keep["router_bias"]),
                                    shared_gate=_lib.ptr(keep["shared_gate"]), shared_up=_lib.ptr(keep["shared_up"]),
                                    shared_down=_lib.ptr(keep["shared_down"]))
        _lib.check(lib.spx_pack_weights(full, src, pk["router_w"].data_ptr(), None, None, _lib.ptr(pk["shared_w1"]),
                                        _lib.ptr(pk["shared_w2"]), stream), "spx_pack_weights (router/shared)")
        self._router_packs[cls] = pk
        return pk

    def _pack_experts(self, rows: int) -> dict:
        from spalmer_b200.experts import SMALL_BATCH_TOKENS

        cls = rows <= SMALL_BATCH_TOKENS
        if cls in self._expert_packs:
            return self._expert_packs[cls]
        lib = _lib.load()
        m, dev = self.mixer, self.device
        stream = torch.cuda.current_stream(dev).cuda_stream
        sl = slice(self.e0, self.e0 + self.e_local)
        gate = m.experts.gate_proj.detach()[sl].contiguous()
        up = m.experts.up_proj.detach()[sl].contiguous()
        down = m.experts.down_proj.detach()[sl].contiguous()
        local = self._local_dims(rows)
        lsizes = _lib.PackedSizes()
        _lib.check(lib.spx_layer_sizes(local, None, lsizes), "spx_layer_sizes")
        empty = lambda n: torch.empty(max(1, n), dtype=torch.int16, device=dev)  # noqa: E731
        pk = {"w1": empty(lsizes.expert_w1), "w2": empty(lsizes.expert_w2), "mx": {}}
        dummy_router = torch.zeros(self.e_local, self.d, dtype=torch.bfloat16, device=dev)
        esrc = _lib.ReferenceWeights(router_weight=dummy_router.data_ptr(), gate_proj=gate.data_ptr(),
                                     up_proj=up.data_ptr(), down_proj=down.data_ptr())
        scratch_router = empty(lsizes.router_weight)
        _lib.check(lib.spx_pack_weights(local, esrc, scratch_router.data_ptr(), pk["w1"].data_ptr(),
                                        pk["w2"].data_ptr(), None, None, stream), "spx_pack_weights (experts)")
        if local.mxfp8_lane:
            from spalmer_b200.experts import pack_lowp_experts

            pk["mx"] = pack_lowp_experts(local, esrc, lsizes, lambda n: torch.empty(n, dtype=torch.uint8, device=dev),
                                         stream)
        pk["keep"] = (gate, up, down, dummy_router, scratch_router)
        self._expert_packs[cls] = pk
        return pk

    def _weights(self, tokens: int, rows: int, lanes: Tensor | None = None) -> _lib.PackedWeights:
        rs = self._pack_router_shared(tokens)
        ex = self._pack_experts(rows)
        mx = ex["mx"]
        return _lib.PackedWeights(
            router_weight=rs["router_w"].data_ptr(), router_bias=_lib.ptr(rs["keep"]["router_bias"]),
            expert_w1=ex["w1"].data_ptr(), expert_w2=ex["w2"].data_ptr(),
            shared_w1=_lib.ptr(rs["shared_w1"]), shared_w2=_lib.ptr(rs["shared_w2"]),
            softplus_table=_lib.ptr(self.lut), resident_mask=None,
            expert_lane_mxfp8=_lib.ptr(lanes),
            expert_w1_mx=_lib.ptr(mx.get("expert_w1_mx")),
            expert_w1_mx_scales=_lib.ptr(mx.get("expert_w1_mx_scales")),
            expert_w2_mx=_lib.ptr(mx.get("expert_w2_mx")),
            expert_w2_mx_scales=_lib.ptr(mx.get("expert_w2_mx_scales")),
            expert_nvfp4_amax=_lib.ptr(mx.get("expert_nvfp4_amax")),
        )

    def _workspace(self, dims: _lib.LayerDims, tag: str) -> Tensor:
        lib = _lib.load()
        n = _lib.ctypes.c_size_t()
        _lib.check(lib.spx_layer_sizes(dims, n, None), "spx_layer_sizes")
        ws = self._ws.get(tag)
        if ws is None or ws.numel() < n.value:
            ws = torch.zeros(n.value, dtype=torch.uint8, device=self.device)
            self._ws[tag] = ws
        return ws

    # ---- stages
    def route(self, x: Tensor, router_logits: Tensor | None = None) -> dict[str, Tensor]:
        lib = _lib.load()
        T = x.shape[0]
        E, k, dev = self.E, self.k, self.device
        dims = self._layer_dims(self.config, T, k)
        ws = self._workspace(dims, "route")
        r = {
            "router_scores": torch.empty(T, E, dtype=torch.bfloat16, device=dev),
            "expert_ids": torch.empty(T, k, dtype=torch.long, device=dev),
            "routing_weights": torch.empty(T, k, dtype=torch.bfloat16, device=dev),
            "expert_utilization": torch.empty(E, dtype=torch.float32, device=dev),
            "group_stats": torch.empty(6, dtype=torch.long, device=dev),
            "group_ratios": torch.empty(2, dtype=torch.float32, device=dev),
            "auxiliary_loss": torch.empty(1, dtype=torch.bfloat16, device=dev),
            "order": torch.empty(T * k, dtype=torch.int32, device=dev),
            "counts": torch.empty(E, dtype=torch.int32, device=dev),
            "rank": torch.empty(T * k, dtype=torch.int32, device=dev),
        }
        outs = _lib.LayerOutputs(
            router_scores=r["router_scores"].data_ptr(), expert_ids=r["expert_ids"].data_ptr(),
            routing_weights=r["routing_weights"].data_ptr(), expert_utilization=r["expert_utilization"].data_ptr(),
            group_stats=r["group_stats"].data_ptr(), group_ratios=r["group_ratios"].data_ptr(),
            auxiliary_loss=r["auxiliary_loss"].data_ptr(), dispatch_order=r["order"].data_ptr(),
            expert_counts=r["counts"].data_ptr(), injected_logits=_lib.ptr(router_logits),
            pair_rank=r["rank"].data_ptr(),
        )
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(lib.spx_layer_route(dims, self._weights(T, 1), x.data_ptr(), outs, ws.data_ptr(), stream),
                   "spx_layer_route")
        return r

    def gather(self, x: Tensor, order: Tensor, div: int) -> Tensor:
        lib = _lib.load()
        out = torch.empty(order.numel(), x.shape[1], dtype=x.dtype, device=x.device)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(lib.spx_gather_rows(x.data_ptr(), x.stride(0), order.data_ptr(), div, order.numel(), x.shape[1],
                                       out.data_ptr(), out.stride(0), stream), "spx_gather_rows")
        return out

    def experts_rows(self, row_ptrs: Tensor, row_expert: Tensor, row_out: Tensor) -> None:
        """BF16 experts whose input row i is read at ``row_ptrs[i]`` and whose
        output row i is stored at ``row_out[i]`` (int64 device tables; peer
        GPUs' memory included)."""

        R = row_ptrs.shape[0]
        if R == 0:
            return
        lib = _lib.load()
        dims = self._local_dims(R)
        ws = self._workspace(dims, "experts")
        stream = torch.cuda.current_stream(row_ptrs.device).cuda_stream
        _lib.check(lib.spx_experts_forward_rows(dims, self._weights(R, R, None), row_ptrs.data_ptr(),
                                                row_expert.data_ptr(), row_out.data_ptr(), ws.data_ptr(), stream),
                   "spx_experts_forward_rows")

    def experts_to(self, rows: Tensor, row_expert: Tensor, lanes: Tensor | None, row_out: Tensor) -> None:
        """Expert outputs of ``rows``, output row i stored by the down
        projection's epilogue at the row pointer ``row_out[i]`` (int64, device;
        a peer GPU's memory included)."""

        R = rows.shape[0]
        if R == 0:
            return
        lib = _lib.load()
        dims = self._local_dims(R)
        ws = self._workspace(dims, "experts")
        stream = torch.cuda.current_stream(rows.device).cuda_stream
        _lib.check(lib.spx_experts_forward_to(dims, self._weights(R, R, lanes), rows.data_ptr(), row_expert.data_ptr(),
                                              row_out.data_ptr(), ws.data_ptr(), stream), "spx_experts_forward_to")

    def experts(self, rows: Tensor, row_expert: Tensor, lanes: Tensor | None, *,
                sorted_out: bool = False) -> Tensor | tuple[Tensor, Tensor]:
        """Expert outputs of ``rows`` in input order, or (``sorted_out``) the
        outputs in dispatch order with each input row's dispatch position, views
        of the workspace valid until its next use."""

        R = rows.shape[0]
        if R == 0:
            empty = torch.empty_like(rows)
            return (empty, torch.empty(0, dtype=torch.int32, device=rows.device)) if sorted_out else empty
        out = None if sorted_out else torch.empty_like(rows)
        lib = _lib.load()
        dims = self._local_dims(R)
        ws = self._workspace(dims, "experts")
        stream = torch.cuda.current_stream(rows.device).cuda_stream
        _lib.check(lib.spx_experts_forward(dims, self._weights(R, R, lanes), rows.data_ptr(), row_expert.data_ptr(),
                                           _lib.ptr(out), ws.data_ptr(), stream), "spx_experts_forward")
        if not sorted_out:
            return out
        y, rank = _lib.ctypes.c_void_p(), _lib.ctypes.c_void_p()
        _lib.check(lib.spx_experts_sorted_rows(dims, ws.data_ptr(), _lib.ctypes.byref(y), _lib.ctypes.byref(rank)),
                   "spx_experts_sorted_rows")
        yv = torch.as_tensor(_RawRows(y.value, R, self.d), device=rows.device).view(torch.bfloat16)
        rv = torch.as_tensor(_RawRows(rank.value, R, 0, "<i4"), device=rows.device)
        return yv, rv

    def shared(self, x: Tensor) -> Tensor | None:
        if self.mixer.shared is None:
            return None
        lib = _lib.load()
        dims = self._layer_dims(self.config, x.shape[0], self.k)
        ws = self._workspace(dims, "shared")
        out = torch.empty_like(x)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(lib.spx_shared_forward(dims, self._weights(x.shape[0], 1), x.data_ptr(), out.data_ptr(),
                                          ws.data_ptr(), stream),
                   "spx_shared_forward")
        return out

    def combine(self, rows: Tensor, rank: Tensor, weights: Tensor | None, shared: Tensor | None,
                tokens: int | None = None) -> Tensor:
        """Per token the sum of its slots' rows (weighted when weights are
        given) on top of `shared`; `rank` is [tokens, slots], -1 = empty."""

        lib = _lib.load()
        T = weights.shape[0] if tokens is None else tokens
        k = rank.numel() // max(T, 1)
        out = torch.empty(T, self.d, dtype=torch.bfloat16, device=rank.device)
        stream = torch.cuda.current_stream(rank.device).cuda_stream
        _lib.check(lib.spx_combine(rows.data_ptr(), rank.data_ptr(), _lib.ptr(weights), _lib.ptr(shared), T, self.d,
                                   k, out.data_ptr(), stream), "spx_combine")
        return out


class _RawRows:
    """A raw device allocation seen by torch as a matrix (zero copy)."""

    def __init__(self, ptr: int, rows: int, cols: int, typestr: str = "<i2"):
        shape = (rows, cols) if cols else (rows,)
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """Exchange buffers of every rank of the group, opened as peer pointers.

    Each rank owns a receive buffer (rows of the pairs routed to its experts,
    from every sender) and a return buffer (the expert outputs of its own
    pairs, in its dispatch order), allocated by ``spx_ipc_buffer_alloc``;
    the CUDA IPC handles are all-gathered once and opened by the peers.  Rows
    move with ``spx_rows_to_peers`` (the sending GPU stores into the peer's
    buffer over NVLink); a one-element NCCL all-reduce after each move orders
    the receivers' reads.  Buffers grow together (the sizes are computed from
    the all-gathered counts, so every rank takes the same decision).
    """

    def __init__(self, group: Any, device: torch.device, d: int):
        self.group = group
        self.device = device
        self.d = d
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.capacity = {"recv": 0, "back": 0}
        self.local: dict[str, int] = {}
        self.peers: dict[str, list[int]] = {}
        self.ptr_tables: dict[str, Tensor] = {}
        self.flag = torch.zeros(1, dtype=torch.int32, device=device)

    def _release(self, kind: str) -> None:
        lib = _lib.load()
        if kind not in self.local:
            return
        torch.cuda.synchronize(self.device)
        self.barrier()
        torch.cuda.synchronize(self.device)  # no peer touches the buffers any more
        for g, ptr in enumerate(self.peers[kind]):
            if g != self.rank:
                _lib.check(lib.spx_ipc_buffer_close(_lib.ctypes.c_void_p(ptr)), "spx_ipc_buffer_close")
        _lib.check(lib.spx_ipc_buffer_free(_lib.ctypes.c_void_p(self.local[kind])), "spx_ipc_buffer_free")
        del self.local[kind], self.peers[kind], self.ptr_tables[kind]
        self.capacity[kind] = 0

    def view_int32(self, kind: str, n: int) -> Tensor:
        """This rank's buffer's first ``n`` int32 values."""

        return torch.as_tensor(_RawRows(self.local[kind], max(n, 0), 0, "<i4"), device=self.device)

    def ensure(self, kind: str, rows: int) -> None:
        """Collective: every rank calls with the same ``rows`` (the largest need),
        in rows of d_model BF16 values."""

        if rows <= self.capacity.get(kind, 0):
            return
        lib = _lib.load()
        self._release(kind)
        cap = max(int(rows * 1.25), 1024)
        ptr = _lib.ctypes.c_void_p()
        handle = (_lib.ctypes.c_uint8 * 64)()
        with torch.cuda.device(self.device):
            _lib.check(lib.spx_ipc_buffer_alloc(cap * self.d * 2, _lib.ctypes.byref(ptr), handle),
                       "spx_ipc_buffer_alloc")
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        allh = torch.empty(self.world * 64, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(allh, mine, group=self.group)
        allh = allh.cpu().numpy().reshape(self.world, 64)
        peers = []
        for g in range(self.world):
            if g == self.rank:
                peers.append(ptr.value)
                continue
            pp = _lib.ctypes.c_void_p()
            h = (_lib.ctypes.c_uint8 * 64)(*allh[g].tolist())
            with torch.cuda.device(self.device):
                _lib.check(lib.spx_ipc_buffer_open(h, _lib.ctypes.byref(pp)), "spx_ipc_buffer_open")
            peers.append(pp.value)
        self.local[kind] = ptr.value
        self.peers[kind] = peers
        self.ptr_tables[kind] = torch.tensor(peers, dtype=torch.int64, device=self.device)
        self.capacity[kind] = cap

    def view(self, kind: str, rows: int) -> Tensor:
        """This rank's buffer rows [0, rows) as a BF16 tensor."""

        raw = torch.as_tensor(_RawRows(self.local[kind], max(rows, 0), self.d), device=self.device)
        return raw.view(torch.bfloat16)

    def send(self, kind: str, src: Tensor, index: Tensor | None, div: int, seg: np.ndarray,
             dst_rows: np.ndarray) -> None:
        """Rows of ``src`` (through ``index // div`` when given) in segments
        ``seg`` [G+1] to every rank's ``kind`` buffer at rows ``dst_rows`` [G]."""

        lib = _lib.load()
        rows = int(seg[-1])
        meta = torch.from_numpy(np.concatenate([seg, dst_rows]).astype(np.int64)).pin_memory()
        meta = meta.to(self.device, non_blocking=True)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(lib.spx_rows_to_peers(src.data_ptr(), src.stride(0), _lib.ptr(index), div, rows, self.d,
                                         meta.data_ptr(), self.ptr_tables[kind].data_ptr(),
                                         meta[self.world + 1:].data_ptr(), self.d, self.world, stream),
                   "spx_rows_to_peers")

    def barrier(self) -> None:
        dist.all_reduce(self.flag, group=self.group)

    def close(self) -> None:
        for kind in list(self.local):
            self._release(kind)


class ExpertParallelMixer:
    """Expert-parallel forward of a `B200MicroExpertChannelMixer` (same
    parameters on every rank; rank r executes experts [r*E/G, (r+1)*E/G)).

    ``forward(hidden [B, S, d])`` takes this rank's tokens and returns their
    update and this rank's routing metrics (statistics over the local tokens).
    ``exchange="peer"`` (the default on CUDA) moves the rows with stores into
    the peers' buffers (``PeerExchange``); ``"nccl"`` with NCCL all-to-all-v.
    """

    def __init__(self, mixer: Any, group: Any = None, ops: Any = None, dedup: bool = False,
                 exchange: str | None = None, peer_rows: str = "store"):
        self.mixer = mixer
        self.dedup = dedup
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.e_local = experts_per_rank(mixer.config.num_experts, self.world)
        if ops is None:
            device = next(mixer.parameters()).device
            ops = CudaOps(mixer, self.rank, self.world, device)
        self.ops = ops
        cuda = isinstance(ops, CudaOps)
        self.side = torch.cuda.Stream(ops.device) if cuda else None
        if exchange is None:
            exchange = "peer" if cuda and not dedup else "nccl"
        if exchange not in {"peer", "nccl"}:
            raise ValueError("exchange must be 'peer' or 'nccl'")
        if exchange == "peer" and (not cuda or dedup):
            raise ValueError("the peer exchange needs the CUDA backend and runs without row de-dup")
        if peer_rows not in {"store", "load"}:
            raise ValueError("peer_rows must be 'store' or 'load'")
        self.exchange = exchange
        self.peer_rows = peer_rows
        self.peer = PeerExchange(group, ops.device, mixer.config.d_model) if exchange == "peer" else None
        self._marks: list | None = None

    def record_stages(self, on: bool) -> None:
        """Record a CUDA event on the compute stream at every stage boundary of
        the next forwards (route, counts + host read, rows out, experts + rows
        back, combine); `stage_times()` returns the mean milliseconds per stage."""

        self._marks = [] if on else None

    def _mark(self, name: str) -> None:
        if self._marks is not None and isinstance(self.ops, CudaOps):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.ops.device))
            self._marks.append((name, ev))

    def stage_times(self) -> dict[str, float]:
        if not self._marks:
            return {}
        torch.cuda.synchronize(self.ops.device)
        sums: dict[str, float] = {}
        calls = 0
        prev = None
        for name, ev in self._marks:
            if name == "start":
                calls += 1
            elif prev is not None:
                sums[name] = sums.get(name, 0.0) + prev.elapsed_time(ev)
            prev = ev
        return {name: v / max(calls, 1) for name, v in sums.items()}

    def close(self) -> None:
        """Release the peer exchange buffers (collective)."""

        if self.peer is not None:
            self.peer.close()

    def _local_lanes(self) -> Tensor | None:
        lanes = self.mixer._lanes(self.ops.device) if isinstance(self.ops, CudaOps) else None
        if lanes is None:
            return None
        return lanes[self.rank * self.e_local:(self.rank + 1) * self.e_local].contiguous()

    def forward(self, hidden: Tensor, *, router_logits: Tensor | None = None) -> dict[str, Any]:
        B, S, d = hidden.shape
        T = B * S
        x = hidden.reshape(T, d).contiguous()
        ops = self.ops
        k = self.mixer.active_experts
        shared = None
        self._mark("start")
        if self.side is not None:
            # the shared SwiGLU needs only x: run it while the rows travel
            self.side.wait_stream(torch.cuda.current_stream(ops.device))
            with torch.cuda.stream(self.side):
                shared = ops.shared(x)
        else:
            shared = ops.shared(x)
        logits = None if router_logits is None else router_logits.reshape(T, -1).contiguous()
        r = ops.route(x, logits)
        self._mark("route")
        if self.dedup:
            update, stats = self._exchange_dedup(x, r, shared)
            return {
                "update": update.reshape(B, S, d),
                "auxiliary_loss": r["auxiliary_loss"][0],
                "expert_ids": r["expert_ids"].reshape(B, S, k),
                "routing_weights": r["routing_weights"].reshape(B, S, k),
                "router_scores": r["router_scores"].reshape(B, S, -1),
                "expert_utilization": r["expert_utilization"],
                **stats,
            }
        if self.peer is not None:
            update, stats = self._exchange_peer(x, r, shared)
            return {
                "update": update.reshape(B, S, d),
                "auxiliary_loss": r["auxiliary_loss"][0],
                "expert_ids": r["expert_ids"].reshape(B, S, k),
                "routing_weights": r["routing_weights"].reshape(B, S, k),
                "router_scores": r["router_scores"].reshape(B, S, -1),
                "expert_utilization": r["expert_utilization"],
                **stats,
            }
        # 2. counts exchange; the only host read of the forward
        recv_counts = torch.empty(self.world * self.e_local, dtype=torch.int32, device=r["counts"].device)
        dist.all_to_all_single(recv_counts, r["counts"], group=self.group)
        plan = exchange_plan(r["counts"].cpu().numpy(), recv_counts.cpu().numpy(), self.world)
        self._mark("counts_alltoall_host_read")
        # 3. rows to their experts' ranks
        send = ops.gather(x, r["order"], k)
        recv = send.new_empty(sum(plan.recv_rows), d)
        dist.all_to_all_single(recv, send, output_split_sizes=plan.recv_rows, input_split_sizes=plan.send_rows,
                               group=self.group)
        self._mark("rows_out")
        # 4. local experts, unweighted
        row_expert = receive_expert_ids(plan, recv.device)
        out_rows = ops.experts(recv, row_expert, self._local_lanes())
        self._mark("experts")
        # 5. back to the senders (in their dispatch order)
        back = send.new_empty(T * k, d)
        dist.all_to_all_single(back, out_rows, output_split_sizes=plan.send_rows, input_split_sizes=plan.recv_rows,
                               group=self.group)
        self._mark("rows_back")
        # 6. combine with the routing weights and the shared output
        if self.side is not None:
            torch.cuda.current_stream(ops.device).wait_stream(self.side)
            if shared is not None:
                shared.record_stream(torch.cuda.current_stream(ops.device))
        update = ops.combine(back, r["rank"], r["routing_weights"], shared)
        self._mark("shared_wait_combine")
        return {
            "update": update.reshape(B, S, d),
            "auxiliary_loss": r["auxiliary_loss"][0],
            "expert_ids": r["expert_ids"].reshape(B, S, k),
            "routing_weights": r["routing_weights"].reshape(B, S, k),
            "router_scores": r["router_scores"].reshape(B, S, -1),
            "expert_utilization": r["expert_utilization"],
            "send_rows": plan.send_rows,
            "recv_rows": plan.recv_rows,
        }

    def _exchange_peer(self, x: Tensor, r: dict, shared: Tensor | None) -> tuple[Tensor, dict]:
        """Steps 2-6 with the rows stored straight into the peers' buffers.

        The all-gathered per-expert counts give every rank the full matrix
        C[s, g] (pairs of rank s on rank g's experts), hence every offset:
        rank s's pairs for g land at rows sum_{s' < s} C[s', g] of g's receive
        buffer, and g returns them to rows sum_{g' < g} C[s, g'] of s's return
        buffer -- s's own dispatch order, which the combine reads.
        """

        ops, G, el, me, k = self.ops, self.world, self.e_local, self.rank, self.mixer.active_experts
        T, d = x.shape
        counts_all = torch.empty(G * self.mixer.config.num_experts, dtype=torch.int32, device=x.device)
        dist.all_gather_into_tensor(counts_all, r["counts"], group=self.group)
        ca = counts_all.cpu().numpy().astype(np.int64).reshape(G, G, el)  # [sender, owner, local expert]
        C = ca.sum(axis=2)  # [sender, owner]
        self._mark("counts_allgather_host_read")
        peer = self.peer
        dev = x.device
        lanes = self._local_lanes()
        # peer_rows="load": BF16 experts' gate/up GEMM gathers its rows straight
        # from the senders' memory (an MXFP8/NVFP4 lane quantises rows it holds,
        # so those rows are always sent first).  "store" (the default) has the
        # senders store the rows into the owners' receive buffers first: on
        # ep_skew at 2 GPUs 4.44 ms per step against 5.31 ms for the GEMM's
        # NVLink gathers, whose latency its producer warp does not hide.
        rows_in_place = self.peer_rows == "load" and lanes is None and d % 64 == 0
        peer.ensure("back", int(C.sum(axis=1).max()))
        R = int(C[:, me].sum())
        plan = ExchangePlan(send_rows=[int(v) for v in C[me]], recv_rows=[int(v) for v in C[:, me]],
                            recv_expert_counts=ca[:, me, :])
        recv_seg = np.concatenate([[0], np.cumsum(C[:, me])])
        back_at = C[:, :me].sum(axis=1)  # = where each sender's pairs for this rank start in its dispatch order
        if rows_in_place:
            # 3. publish this rank's rows and dispatch order; every owner gathers from them
            peer.ensure("x", int(C.sum(axis=1).max()) // k + 1)
            peer.ensure("order", (int(C.sum(axis=1).max()) * 4 + 2 * d - 1) // (2 * d))
            peer.view("x", T).copy_(x)
            peer.view_int32("order", T * k).copy_(r["order"])
            peer.barrier()
        else:
            # 3. rows of this rank's pairs (dispatch order) -> owners' receive buffers
            peer.ensure("recv", int(C.sum(axis=0).max()))
            send_seg = np.concatenate([[0], np.cumsum(C[me])])
            recv_at = C[:me].sum(axis=0)  # where this rank's block starts in every owner's buffer
            peer.send("recv", x, r["order"], k, send_seg, recv_at)
            peer.barrier()
        self._mark("rows_out")
        # 4-5. local experts; the down projection's epilogue stores received row i's
        #      output straight into its sender's return buffer, at the row of the
        #      sender's dispatch order
        if R:
            src = torch.repeat_interleave(torch.arange(G, device=dev),
                                          torch.from_numpy(np.ascontiguousarray(C[:, me])).to(dev))
            rows_at = torch.from_numpy(back_at - recv_seg[:-1]).to(dev)[src] + torch.arange(R, device=dev)
            row_out = peer.ptr_tables["back"][src] + rows_at * (d * 2)
            row_expert = receive_expert_ids(plan, dev)
            if rows_in_place:
                lib = _lib.load()
                meta = torch.from_numpy(np.concatenate([back_at, recv_seg]).astype(np.int64)).to(dev)
                row_ptrs = torch.empty(R, dtype=torch.int64, device=dev)
                _lib.check(lib.spx_peer_row_pointers(peer.ptr_tables["order"].data_ptr(), meta.data_ptr(),
                                                     meta[G:].data_ptr(), G, k, peer.ptr_tables["x"].data_ptr(),
                                                     d, R, row_ptrs.data_ptr(),
                                                     torch.cuda.current_stream(dev).cuda_stream),
                           "spx_peer_row_pointers")
                ops.experts_rows(row_ptrs, row_expert, row_out)
            else:
                ops.experts_to(peer.view("recv", R), row_expert, lanes, row_out)
        peer.barrier()
        self._mark("experts_rows_back")
        # 6. combine with the routing weights and the shared output
        if self.side is not None:
            torch.cuda.current_stream(ops.device).wait_stream(self.side)
            if shared is not None:
                shared.record_stream(torch.cuda.current_stream(ops.device))
        update = ops.combine(peer.view("back", T * k), r["rank"], r["routing_weights"], shared)
        self._mark("shared_wait_combine")
        return update, {"send_rows": plan.send_rows, "recv_rows": plan.recv_rows}

    def _exchange_dedup(self, x: Tensor, r: dict, shared: Tensor | None) -> tuple[Tensor, dict]:
        """The exchange with token rows sent once per destination rank.

        A token whose k pairs land on m experts of one rank travels to that
        rank once instead of m times; with each pair goes a 64-bit word (the
        token's row within the destination's block << 16 | its BF16 routing
        weight).  The destination expands the rows to its pairs, runs its
        experts, and sums each token's weighted pair rows (one BF16 row per
        token and destination) before sending them back; the source adds those
        to the shared output.  Per token the pair rows are summed per
        destination first, so the update matches the single-GPU layer within
        BF16 tolerance rather than bit for bit.
        """

        ops, G, el, k = self.ops, self.world, self.e_local, self.mixer.active_experts
        T, d = x.shape
        dev = x.device
        order = r["order"].long()
        counts = r["counts"].long()
        # sorted pairs are grouped by expert, hence by destination rank
        dest_sorted = torch.repeat_interleave(torch.arange(G, device=dev), counts.view(G, el).sum(1))
        key = dest_sorted * T + order // k
        uniq, inv = torch.unique(key, sorted=True, return_inverse=True)
        uniq_dest = uniq // T
        uniq_tok = uniq % T
        uniq_counts = torch.bincount(uniq_dest, minlength=G)
        uniq_off = torch.cumsum(uniq_counts, 0) - uniq_counts
        rel = inv - uniq_off[dest_sorted]
        # 2. per destination: pair counts of its experts and the unique rows; one host read
        send_meta = torch.cat([counts.view(G, el), uniq_counts.view(G, 1)], dim=1).to(torch.int32).contiguous()
        recv_meta = torch.empty_like(send_meta)
        dist.all_to_all_single(recv_meta, send_meta, group=self.group)
        sm, rm = send_meta.cpu().numpy(), recv_meta.cpu().numpy()
        plan = exchange_plan(sm[:, :el].reshape(-1), rm[:, :el].reshape(-1), G)
        send_u = [int(v) for v in sm[:, el]]
        recv_u = [int(v) for v in rm[:, el]]
        # 3. unique rows out, and the pairs' (row, weight) words
        send_rows = ops.gather(x, uniq_tok.to(torch.int32), 1)
        recv_rows = send_rows.new_empty(sum(recv_u), d)
        dist.all_to_all_single(recv_rows, send_rows, output_split_sizes=recv_u, input_split_sizes=send_u,
                               group=self.group)
        w_sorted = r["routing_weights"].reshape(-1)[order].contiguous()
        words = (rel << 16) | (w_sorted.view(torch.int16).to(torch.int64) & 0xFFFF)
        recv_words = words.new_empty(sum(plan.recv_rows))
        dist.all_to_all_single(recv_words, words, output_split_sizes=plan.recv_rows,
                               input_split_sizes=plan.send_rows, group=self.group)
        # 4. expand to pair rows, local experts (unweighted)
        recv_u_t = torch.tensor(recv_u, dtype=torch.int64, device=dev)
        src_of_pair = torch.repeat_interleave(torch.arange(G, device=dev),
                                              torch.tensor(plan.recv_rows, dtype=torch.int64, device=dev))
        row_index = (torch.cumsum(recv_u_t, 0) - recv_u_t)[src_of_pair] + (recv_words >> 16)
        w_recv = (recv_words & 0xFFFF).to(torch.int16).view(torch.bfloat16)
        pair_rows = ops.gather(recv_rows, row_index.to(torch.int32).contiguous(), 1)
        out_rows = ops.experts(pair_rows, receive_expert_ids(plan, dev), self._local_lanes())
        # 5. per received row, the sum of its pairs' bf16(row * weight): a slot table [U, k]
        U, P = recv_rows.shape[0], out_rows.shape[0]
        perm = torch.argsort(row_index, stable=True)
        cnt = torch.bincount(row_index, minlength=U)
        u_sorted = row_index[perm]
        slot = torch.arange(P, device=dev) - (torch.cumsum(cnt, 0) - cnt)[u_sorted]
        table = torch.full((U * k,), -1, dtype=torch.int32, device=dev)
        table[u_sorted * k + slot] = perm.to(torch.int32)
        wtab = torch.zeros(U * k, dtype=torch.bfloat16, device=dev)
        wtab[u_sorted * k + slot] = w_recv[perm]
        partial = (ops.combine(out_rows, table, wtab.view(U, k), None, tokens=U) if U > 0
                   else out_rows.new_empty(0, d))
        back = partial.new_empty(sum(send_u), d)
        dist.all_to_all_single(back, partial, output_split_sizes=send_u, input_split_sizes=recv_u,
                               group=self.group)
        # 6. update = shared + the partial rows of every destination (slot = destination rank)
        if self.side is not None:
            torch.cuda.current_stream(ops.device).wait_stream(self.side)
            if shared is not None:
                shared.record_stream(torch.cuda.current_stream(ops.device))
        tab2 = torch.full((T * G,), -1, dtype=torch.int32, device=dev)
        tab2[uniq_tok * G + uniq_dest] = torch.arange(uniq.numel(), dtype=torch.int32, device=dev)
        update = ops.combine(back, tab2, None, shared, tokens=T)
        return update, {"send_rows": send_u, "recv_rows": recv_u, "send_pairs": plan.send_rows,
                        "recv_pairs": plan.recv_rows}

    __call__ = forward


__all__ = ["CudaOps", "ExchangePlan", "ExpertParallelMixer", "PeerExchange", "exchange_plan", "experts_per_rank",
           "receive_expert_ids"]
