"""libspx loads on the CPU host and exports every symbol include/spx.h declares."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from spalmer_b200 import _lib
from spalmer_b200.build import TARGET, build

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> set[str]:
    text = (ROOT / "include" / "spx.h").read_text()
    return set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(spx_\w+)\s*\(", text, flags=re.M))


def test_library_builds_and_loads():
    build()
    assert TARGET.exists()
    lib = _lib.load()
    assert lib.spx_abi_version() == _lib.ABI_VERSION == 12


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(TARGET))
    declared = declared_functions()
    assert declared, "no declarations parsed from include/spx.h"
    assert declared == set(_lib.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name


def test_status_strings_and_host_only_sizes():
    lib = _lib.load()
    assert lib.spx_status_string(0) == b"ok"
    assert b"invalid" in lib.spx_status_string(-1)
    dims = _lib.LayerDims(tokens=65536, d_model=768, num_experts=200, inter_dim=128, shared_dim=768,
                          top_k=8, score_transform=0, execution_loop=0)
    ws = ctypes.c_size_t()
    sizes = _lib.PackedSizes()
    assert lib.spx_layer_sizes(dims, ws, sizes) == 0
    assert sizes.expert_w1 == 200 * 256 * 768
    assert sizes.expert_w2 == 200 * 768 * 128
    assert sizes.shared_w1 == 2 * 768 * 768
    assert ws.value > 2 * 65536 * 8 * 768  # holds the per-pair expert outputs


@pytest.mark.parametrize(
    "field,value", [("top_k", 0), ("top_k", 21), ("num_experts", 0), ("tokens", 0), ("inter_dim", 0)]
)
def test_invalid_dims_are_rejected(field, value):
    lib = _lib.load()
    kw = dict(tokens=16, d_model=64, num_experts=8, inter_dim=16, shared_dim=0, top_k=2,
              score_transform=0, execution_loop=0)
    kw[field] = value
    dims = _lib.LayerDims(**kw)
    assert lib.spx_layer_sizes(dims, None, None) < 0


def test_null_pointers_are_rejected_without_a_gpu():
    lib = _lib.load()
    dims = _lib.LayerDims(tokens=16, d_model=64, num_experts=8, inter_dim=16, shared_dim=0, top_k=2,
                          score_transform=0, execution_loop=0)
    assert lib.spx_route(dims, None, None, None, None, None, None, None, None) == -1
    assert lib.spx_dispatch(dims, None, None, None, None, None) == -1
    assert lib.spx_layer_forward(dims, None, None, None, None, None) == -1
    assert lib.spx_softplus_table(None, None) == -1
    assert lib.spx_mxfp8_quantize_rows(None, 4, 32, None, None, None) == -1
    assert lib.spx_mxfp8_quantize_rows(None, 4, 37, None, None, None) == -1  # cols % 32 != 0
    assert lib.spx_mxfp8_mm_nt(None, None, 7, 23, 37, None, None, 0, None) == -1


def test_mxfp8_sizes_are_host_only():
    """MXFP8 copies: E4M3 bytes plus 512-byte scale atoms (128 rows x 4 blocks of 32)."""

    lib = _lib.load()
    dims = _lib.LayerDims(tokens=65536, d_model=768, num_experts=200, inter_dim=128, shared_dim=768,
                          top_k=8, score_transform=0, execution_loop=0, mxfp8_lane=1)
    ws_mx = ctypes.c_size_t()
    sizes = _lib.PackedSizes()
    assert lib.spx_layer_sizes(dims, ws_mx, sizes) == 0
    assert sizes.expert_w1_mx == 200 * 256 * 768
    assert sizes.expert_w1_mx_scales == 200 * 2 * (768 // 128) * 512  # two 128-row tiles of [gate|up]
    assert sizes.expert_w2_mx == 200 * 768 * 128
    assert sizes.expert_w2_mx_scales == 200 * 6 * 1 * 512
    dims.mxfp8_lane = 0
    ws = ctypes.c_size_t()
    assert lib.spx_layer_sizes(dims, ws, sizes) == 0
    assert sizes.expert_w1_mx == 0
    # quantised hidden states [T, d] + hidden rows [P, I] and their scales
    assert ws_mx.value - ws.value >= 65536 * 768 + 65536 * 8 * 128
    # I % 32 != 0 has no MXFP8 lane
    dims = _lib.LayerDims(tokens=16, d_model=64, num_experts=8, inter_dim=48, shared_dim=0, top_k=2,
                          score_transform=0, execution_loop=0, mxfp8_lane=1)
    assert lib.spx_layer_sizes(dims, None, None) == -2
    assert lib.spx_mxfp8_mm_workspace(7, 23, 37) > 7 * 128 + 23 * 128
