"""ctypes binding of libspx (the C ABI declared in ``include/spx.h``).

The shared library is built in-tree by ``spalmer_b200.build`` and loaded from
``spalmer_b200/libspx.so``.  There is no fallback: if the library is missing
or fails to load, every GPU entry point raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libspx.so"

SPX_OK = 0
STATUS_NAMES = {
    -1: "SPX_ERR_INVALID_ARG",
    -2: "SPX_ERR_UNSUPPORTED",
    -3: "SPX_ERR_CUDA",
    -4: "SPX_ERR_DRIVER",
    -5: "SPX_ERR_TIMEOUT",
    -6: "SPX_ERR_ALIGNMENT",
    -7: "SPX_ERR_WORKSPACE",
    -8: "SPX_ERR_DEVICE",
    -9: "SPX_ERR_SCRATCH_LIMIT",
}

# Every function exported by include/spx.h (checked by tests/test_abi_symbols.py).
EXPORTED = (
    "spx_abi_version",
    "spx_status_string",
    "spx_layer_sizes",
    "spx_softplus_table",
    "spx_pack_weights",
    "spx_route",
    "spx_dispatch",
    "spx_layer_forward",
    "spx_workspace_status",
    "spx_dispatch_static",
    "spx_pack_weights_mxfp8",
    "spx_mxfp8_quantize_rows",
    "spx_mxfp8_mm_workspace",
    "spx_mxfp8_mm_nt",
    "spx_layer_route",
    "spx_gather_rows",
    "spx_swiglu_backward_rows",
    "spx_experts_forward",
    "spx_shared_forward",
    "spx_combine",
    "spx_calibration_workspace",
    "spx_surprise_calibration",
    "spx_layer_backward_sizes",
    "spx_layer_saved_gu_cols",
    "spx_layer_saved_shared_gu",
    "spx_layer_backward",
    "spx_block_channel_forward",
    "spx_rmsnorm_rows",
    "spx_expert_quant_error",
    "spx_layer_paged_begin",
    "spx_layer_paged_experts",
    "spx_layer_paged_finish",
    "spx_stage_expert_slots",
    "spx_nvfp4_quantize_rows",
    "spx_nvfp4_mm_workspace",
    "spx_nvfp4_mm_nt",
    "spx_pack_weights_nvfp4",
    "spx_ipc_buffer_alloc",
    "spx_ipc_buffer_open",
    "spx_ipc_buffer_close",
    "spx_ipc_buffer_free",
    "spx_rows_to_peers",
    "spx_experts_sorted_rows",
    "spx_experts_forward_to",
    "spx_experts_forward_rows",
    "spx_peer_row_pointers",
    "spx_router_sizes",
    "spx_router_forward",
    "spx_dispatch_static_status",
)

ABI_VERSION = 12

_vp = ctypes.c_void_p


class LayerDims(ctypes.Structure):
    _fields_ = [
        ("tokens", ctypes.c_int64),
        ("d_model", ctypes.c_int32),
        ("num_experts", ctypes.c_int32),
        ("inter_dim", ctypes.c_int32),
        ("shared_dim", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("score_transform", ctypes.c_int32),
        ("execution_loop", ctypes.c_int32),
        ("mxfp8_lane", ctypes.c_int32),
    ]


class ReferenceWeights(ctypes.Structure):
    _fields_ = [
        ("router_weight", _vp),
        ("router_bias", _vp),
        ("gate_proj", _vp),
        ("up_proj", _vp),
        ("down_proj", _vp),
        ("shared_gate", _vp),
        ("shared_up", _vp),
        ("shared_down", _vp),
    ]


class PackedSizes(ctypes.Structure):
    _fields_ = [
        ("router_weight", ctypes.c_size_t),
        ("expert_w1", ctypes.c_size_t),
        ("expert_w2", ctypes.c_size_t),
        ("shared_w1", ctypes.c_size_t),
        ("shared_w2", ctypes.c_size_t),
        ("expert_w1_mx", ctypes.c_size_t),
        ("expert_w1_mx_scales", ctypes.c_size_t),
        ("expert_w2_mx", ctypes.c_size_t),
        ("expert_w2_mx_scales", ctypes.c_size_t),
        ("expert_nvfp4_amax", ctypes.c_size_t),
    ]


class PackedWeights(ctypes.Structure):
    _fields_ = [
        ("router_weight", _vp),
        ("router_bias", _vp),
        ("expert_w1", _vp),
        ("expert_w2", _vp),
        ("shared_w1", _vp),
        ("shared_w2", _vp),
        ("softplus_table", _vp),
        ("resident_mask", _vp),
        ("expert_lane_mxfp8", _vp),
        ("expert_w1_mx", _vp),
        ("expert_w1_mx_scales", _vp),
        ("expert_w2_mx", _vp),
        ("expert_w2_mx_scales", _vp),
        ("expert_nvfp4_amax", _vp),
        ("expert_quant_error", _vp),
    ]


class LayerOutputs(ctypes.Structure):
    _fields_ = [
        ("update", _vp),
        ("router_scores", _vp),
        ("expert_ids", _vp),
        ("routing_weights", _vp),
        ("expert_utilization", _vp),
        ("group_stats", _vp),
        ("group_ratios", _vp),
        ("auxiliary_loss", _vp),
        ("dispatch_order", _vp),
        ("expert_counts", _vp),
        ("injected_logits", _vp),
        ("router_logits", _vp),
        ("stage_events", _vp),
        ("pair_rank", _vp),
        ("expert_quantization_error", _vp),
        ("saved_x", _vp),
        ("saved_gu", _vp),
        ("saved_shared_gu", _vp),
    ]


class LayerGrads(ctypes.Structure):
    _fields_ = [
        ("expert_ids", _vp),
        ("routing_weights", _vp),
        ("router_scores", _vp),
        ("gate_proj", _vp),
        ("up_proj", _vp),
        ("down_proj", _vp),
        ("d_update", _vp),
        ("d_scores", _vp),
        ("d_aux", _vp),
        ("d_hidden_experts", _vp),
        ("d_logits", _vp),
        ("x_sorted", _vp),
        ("h_sorted", _vp),
        ("du_sorted", _vp),
        ("dgu_sorted", _vp),
        ("expert_counts", _vp),
        ("d_gate_proj", _vp),
        ("d_up_proj", _vp),
        ("d_down_proj", _vp),
        ("saved_gu", _vp),
        ("router_logits", _vp),
        ("forward_workspace", _vp),
        ("expert_utilization", _vp),
    ]


STAGE_EVENTS = 8
STAGE_NAMES = ("router_gemm", "route_topk", "dispatch", "expert_gemm1_swiglu", "expert_gemm2_scatter",
               "shared_gemm1_swiglu", "shared_gemm2_combine")


_lib = None


class SpxError(RuntimeError):
    """A libspx entry point returned a non-zero status."""


def load() -> ctypes.CDLL:
    """Load libspx, raising if it is absent (no CPU fallback exists)."""

    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise SpxError(
            f"libspx is not built ({LIB_PATH} missing); run `python -m spalmer_b200.build`"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    P = ctypes.POINTER
    sig = {
        "spx_abi_version": (ctypes.c_int, []),
        "spx_status_string": (ctypes.c_char_p, [ctypes.c_int]),
        "spx_layer_sizes": (ctypes.c_int, [P(LayerDims), P(ctypes.c_size_t), P(PackedSizes)]),
        "spx_softplus_table": (ctypes.c_int, [_vp, _vp]),
        "spx_pack_weights": (
            ctypes.c_int,
            [P(LayerDims), P(ReferenceWeights), _vp, _vp, _vp, _vp, _vp, _vp],
        ),
        "spx_route": (ctypes.c_int, [P(LayerDims), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
        "spx_dispatch": (ctypes.c_int, [P(LayerDims), _vp, _vp, _vp, _vp, _vp]),
        "spx_layer_forward": (
            ctypes.c_int,
            [P(LayerDims), P(PackedWeights), _vp, P(LayerOutputs), _vp, _vp],
        ),
        "spx_workspace_status": (ctypes.c_int, [_vp, P(ctypes.c_int), ctypes.c_int, _vp]),
        "spx_dispatch_static": (ctypes.c_int, [P(LayerDims), _vp, _vp, _vp, _vp]),
        "spx_dispatch_static_status": (ctypes.c_int, [P(ctypes.c_int), ctypes.c_int, _vp]),
        "spx_router_sizes": (ctypes.c_int, [P(LayerDims), P(ctypes.c_size_t)]),
        "spx_router_forward": (ctypes.c_int, [P(LayerDims), P(PackedWeights), _vp, _vp, _vp, _vp]),
        "spx_pack_weights_mxfp8": (ctypes.c_int, [P(LayerDims), P(ReferenceWeights), _vp, _vp, _vp, _vp, _vp]),
        "spx_mxfp8_quantize_rows": (ctypes.c_int, [_vp, ctypes.c_int64, ctypes.c_int32, _vp, _vp, _vp]),
        "spx_mxfp8_mm_workspace": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]),
        "spx_layer_route": (ctypes.c_int, [P(LayerDims), P(PackedWeights), _vp, P(LayerOutputs), _vp, _vp]),
        "spx_gather_rows": (
            ctypes.c_int,
            [_vp, ctypes.c_int64, _vp, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, _vp, ctypes.c_int64, _vp],
        ),
        "spx_swiglu_backward_rows": (
            ctypes.c_int,
            [_vp, ctypes.c_int64, ctypes.c_int32, _vp, ctypes.c_int64, _vp, _vp, ctypes.c_int64, ctypes.c_int32,
             ctypes.c_int32, _vp, _vp, _vp, _vp],
        ),
        "spx_experts_forward": (ctypes.c_int, [P(LayerDims), P(PackedWeights), _vp, _vp, _vp, _vp, _vp]),
        "spx_shared_forward": (ctypes.c_int, [P(LayerDims), P(PackedWeights), _vp, _vp, _vp, _vp]),
        "spx_calibration_workspace": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32]),
        "spx_surprise_calibration": (
            ctypes.c_int,
            [_vp, _vp, _vp, _vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, _vp, _vp, _vp,
             _vp, ctypes.c_size_t, _vp],
        ),
        "spx_combine": (
            ctypes.c_int,
            [_vp, _vp, _vp, _vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, _vp, _vp],
        ),
        "spx_layer_backward_sizes": (ctypes.c_int, [P(LayerDims), P(ctypes.c_size_t)]),
        "spx_layer_saved_gu_cols": (ctypes.c_int, [P(LayerDims), P(ctypes.c_int64)]),
        "spx_layer_saved_shared_gu": (ctypes.c_int, [P(LayerDims), P(ctypes.c_int64), P(ctypes.c_int32)]),
        "spx_layer_backward": (ctypes.c_int, [P(LayerDims), P(PackedWeights), _vp, P(LayerGrads), _vp, _vp]),
        "spx_block_channel_forward": (
            ctypes.c_int,
            [P(LayerDims), P(PackedWeights), _vp, ctypes.c_float, _vp, P(LayerOutputs), _vp, _vp, _vp],
        ),
        "spx_expert_quant_error": (ctypes.c_int, [P(LayerDims), P(ReferenceWeights), ctypes.c_int32, _vp, _vp]),
        "spx_rmsnorm_rows": (
            ctypes.c_int,
            [_vp, _vp, ctypes.c_float, ctypes.c_int64, ctypes.c_int32, _vp, ctypes.c_int32, _vp],
        ),
        "spx_layer_paged_begin": (ctypes.c_int, [P(LayerDims), P(PackedWeights), _vp, P(LayerOutputs), _vp, _vp]),
        "spx_layer_paged_experts": (
            ctypes.c_int,
            [P(LayerDims), P(PackedWeights), ctypes.c_int32, _vp, ctypes.c_int32, _vp, _vp, _vp],
        ),
        "spx_layer_paged_finish": (ctypes.c_int, [P(LayerDims), P(PackedWeights), _vp, P(LayerOutputs), _vp, _vp]),
        "spx_stage_expert_slots": (
            ctypes.c_int,
            [_vp, _vp, _vp, ctypes.c_int32, _vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
             _vp],
        ),
        "spx_nvfp4_quantize_rows": (ctypes.c_int, [_vp, ctypes.c_int64, ctypes.c_int32, _vp, _vp, _vp, _vp]),
        "spx_pack_weights_nvfp4": (ctypes.c_int, [P(LayerDims), P(ReferenceWeights), _vp, _vp, _vp, _vp, _vp, _vp]),
        "spx_ipc_buffer_alloc": (ctypes.c_int, [ctypes.c_size_t, P(_vp), _vp]),
        "spx_ipc_buffer_open": (ctypes.c_int, [_vp, P(_vp)]),
        "spx_ipc_buffer_close": (ctypes.c_int, [_vp]),
        "spx_ipc_buffer_free": (ctypes.c_int, [_vp]),
        "spx_experts_sorted_rows": (ctypes.c_int, [P(LayerDims), _vp, P(_vp), P(_vp)]),
        "spx_experts_forward_to": (ctypes.c_int, [P(LayerDims), P(PackedWeights), _vp, _vp, _vp, _vp, _vp]),
        "spx_experts_forward_rows": (ctypes.c_int, [P(LayerDims), P(PackedWeights), _vp, _vp, _vp, _vp, _vp]),
        "spx_peer_row_pointers": (
            ctypes.c_int,
            [_vp, _vp, _vp, ctypes.c_int32, ctypes.c_int32, _vp, ctypes.c_int64, ctypes.c_int64, _vp, _vp],
        ),
        "spx_rows_to_peers": (
            ctypes.c_int,
            [_vp, ctypes.c_int64, _vp, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, _vp, _vp, _vp, ctypes.c_int64,
             ctypes.c_int32, _vp],
        ),
        "spx_nvfp4_mm_workspace": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]),
        "spx_nvfp4_mm_nt": (
            ctypes.c_int,
            [_vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp, _vp, ctypes.c_size_t, _vp],
        ),
        "spx_mxfp8_mm_nt": (
            ctypes.c_int,
            [_vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp, _vp, ctypes.c_size_t, _vp],
        ),
    }
    for name, (restype, argtypes) in sig.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.spx_abi_version() != ABI_VERSION:
        raise SpxError(f"libspx ABI version {lib.spx_abi_version()} != {ABI_VERSION}")
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != SPX_OK:
        lib = load()
        text = lib.spx_status_string(status).decode()
        raise SpxError(f"{what} failed: {STATUS_NAMES.get(status, status)} ({text})")


def ptr(tensor) -> int | None:
    """Device pointer of a tensor (None for None)."""

    return None if tensor is None else tensor.data_ptr()
