"""Native precision providers on B200 (the reference's experts/native.py surface).

* ``native_provider_capabilities``: the capability hook the reference imports
  (precision.py:396-430), with claims shaped like ``ExpertPrecisionCapability``
  (precision.py:68-107).  Claims are verified by running one small layer on the
  device.  The BF16 pair trains (``spx_layer_backward``); the MXFP8 and NVFP4
  pairs are forward-only, so their ``backward_available`` is False.
* ``mx_quantize_rows`` / ``mxfp8_mm_nt`` / ``native_mxfp8_linear``,
  ``nvfp4_quantize_rows`` / ``nvfp4_mm_nt`` / ``native_nvfp4_linear`` and
  ``native_expert_matmul``: forward-only equivalents of ``_mx_quantize_rows``,
  ``_mxfp8_mm_nt``, ``native_mxfp8_linear``, ``_pack_nvfp4``,
  ``native_nvfp4_linear`` and ``native_expert_matmul`` (experts/native.py:91-350)
  running on libspx's quantisers and block-scaled tcgen05 GEMMs
  (kind::mxf8f6f4 and kind::mxf4nvf4).  No emulation: other pairs raise.
"""

from __future__ import annotations

from functools import lru_cache

import torch
from torch import Tensor

from spalmer_b200 import _lib

PROVIDER_ID = "spx_sm100_grouped"


class NativeExpertPrecisionError(RuntimeError):
    """Raised when a requested native expert kernel cannot execute (experts/native.py:30-31)."""


def _require_cuda_bf16(left: Tensor, right: Tensor, *, operation: str) -> None:
    if not left.is_cuda or not right.is_cuda:
        raise NativeExpertPrecisionError(f"{operation} requires CUDA operands")
    if left.device != right.device:
        raise NativeExpertPrecisionError(f"{operation} operands must share one device")
    if left.dtype != torch.bfloat16 or right.dtype != torch.bfloat16:
        raise NativeExpertPrecisionError(f"{operation} requires BF16 source activations and master weights")


def _forward_only(*tensors: Tensor) -> None:
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors):
        raise NotImplementedError("the B200 low-precision (MXFP8/NVFP4) provider implements the forward pass only")


def mx_quantize_rows(value: Tensor) -> tuple[Tensor, Tensor]:
    """E4M3 values ``[rows, cols]`` and E8M0 scale bytes ``[rows, cols/32]`` (uint8) of BF16 rows."""

    if value.ndim != 2 or value.dtype != torch.bfloat16 or not value.is_cuda:
        raise ValueError("mx_quantize_rows expects a [rows, cols] bfloat16 CUDA tensor")
    rows, cols = value.shape
    if cols % 32:
        raise ValueError("the row length must be a multiple of the block size 32")
    src = value.contiguous()
    values = torch.empty(rows, cols, dtype=torch.uint8, device=value.device)
    scales = torch.empty(rows, cols // 32, dtype=torch.uint8, device=value.device)
    lib = _lib.load()
    stream = torch.cuda.current_stream(value.device).cuda_stream
    _lib.check(lib.spx_mxfp8_quantize_rows(src.data_ptr(), rows, cols, values.data_ptr(), scales.data_ptr(), stream),
               "spx_mxfp8_quantize_rows")
    return values, scales


def mxfp8_mm_nt(left: Tensor, right_rows: Tensor) -> Tensor:
    """``left @ right_rows.T`` with both operands MXFP8 (experts/native.py:113-140)."""

    if left.ndim != 2 or right_rows.ndim != 2:
        raise ValueError("native MXFP8 operands must be rank-2 matrices")
    if left.shape[1] != right_rows.shape[1]:
        raise ValueError("native MXFP8 operands must share a contraction dimension")
    _require_cuda_bf16(left, right_rows, operation="native MXFP8 GEMM")
    _forward_only(left, right_rows)
    m, k = left.shape
    n = right_rows.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=left.device)
    if m == 0 or n == 0:
        return out
    lib = _lib.load()
    nbytes = lib.spx_mxfp8_mm_workspace(m, n, k)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=left.device)
    a = left.detach().contiguous()
    b = right_rows.detach().contiguous()
    stream = torch.cuda.current_stream(left.device).cuda_stream
    _lib.check(lib.spx_mxfp8_mm_nt(a.data_ptr(), b.data_ptr(), m, n, k, out.data_ptr(), ws.data_ptr(), nbytes,
                                   stream), "spx_mxfp8_mm_nt")
    return out


def native_mxfp8_linear(input: Tensor, weight: Tensor, bias: Tensor | None = None) -> Tensor:
    """``F.linear`` whose GEMM executes in MXFP8 (experts/native.py:193-202), forward only."""

    if weight.ndim != 2 or input.ndim < 1 or input.shape[-1] != weight.shape[1]:
        raise ValueError("native MXFP8 linear received incompatible input/weight shapes")
    _require_cuda_bf16(input, weight, operation="native MXFP8 linear")
    out = mxfp8_mm_nt(input.reshape(-1, input.shape[-1]), weight)
    if bias is not None:
        out = out + bias
    return out.reshape(*input.shape[:-1], weight.shape[0])


def nvfp4_quantize_rows(value: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """``_pack_nvfp4`` of BF16 rows (experts/native.py:205-218): E2M1 values
    ``[rows, kp/2]`` (two per byte), UE4M3 scale bytes ``[rows, kp/16]`` and the
    per-tensor amax (float32 scalar; the per-tensor scale is amax / 2688), with
    kp = cols rounded up to 256 (zero columns beyond cols)."""

    if value.ndim != 2 or value.dtype != torch.bfloat16 or not value.is_cuda:
        raise ValueError("nvfp4_quantize_rows expects a [rows, cols] bfloat16 CUDA tensor")
    rows, cols = value.shape
    if cols < 1:
        raise ValueError("the row length must be positive")
    kp = -(-cols // 256) * 256
    src = value.contiguous()
    values = torch.empty(rows, kp // 2, dtype=torch.uint8, device=value.device)
    scales = torch.empty(rows, kp // 16, dtype=torch.uint8, device=value.device)
    amax = torch.zeros((), dtype=torch.float32, device=value.device)
    lib = _lib.load()
    stream = torch.cuda.current_stream(value.device).cuda_stream
    _lib.check(lib.spx_nvfp4_quantize_rows(src.data_ptr(), rows, cols, values.data_ptr(), scales.data_ptr(),
                                           amax.data_ptr(), stream), "spx_nvfp4_quantize_rows")
    return values, scales, amax


def nvfp4_mm_nt(left: Tensor, right_rows: Tensor) -> Tensor:
    """``left @ right_rows.T`` with both operands NVFP4 (experts/native.py:224-262)."""

    if left.ndim != 2 or right_rows.ndim != 2:
        raise ValueError("native NVFP4 operands must be rank-2 matrices")
    if left.shape[1] != right_rows.shape[1]:
        raise ValueError("native NVFP4 operands must share a contraction dimension")
    _require_cuda_bf16(left, right_rows, operation="native NVFP4 GEMM")
    _forward_only(left, right_rows)
    m, k = left.shape
    n = right_rows.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=left.device)
    if m == 0 or n == 0:
        return out
    lib = _lib.load()
    nbytes = lib.spx_nvfp4_mm_workspace(m, n, k)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=left.device)
    a = left.detach().contiguous()
    b = right_rows.detach().contiguous()
    stream = torch.cuda.current_stream(left.device).cuda_stream
    _lib.check(lib.spx_nvfp4_mm_nt(a.data_ptr(), b.data_ptr(), m, n, k, out.data_ptr(), ws.data_ptr(), nbytes,
                                   stream), "spx_nvfp4_mm_nt")
    return out


def native_nvfp4_linear(input: Tensor, weight: Tensor, bias: Tensor | None = None) -> Tensor:
    """``F.linear`` whose GEMM executes in NVFP4 (experts/native.py:292-302), forward only."""

    if weight.ndim != 2 or input.ndim < 1 or input.shape[-1] != weight.shape[1]:
        raise ValueError("native NVFP4 linear received incompatible input/weight shapes")
    _require_cuda_bf16(input, weight, operation="native NVFP4 linear")
    out = nvfp4_mm_nt(input.reshape(-1, input.shape[-1]), weight)
    if bias is not None:
        out = out + bias
    return out.reshape(*input.shape[:-1], weight.shape[0])


def native_expert_matmul(input: Tensor, weight: Tensor, bias: Tensor | None = None, *, weight_format: str,
                         activation_format: str) -> Tensor:
    """``input @ weight`` for an expert's ``[in, out]`` weight (experts/native.py:305-350).

    The ("mxfp8", "mxfp8") and ("nvfp4", "nvfp4") pairs run here; the BF16
    expert lane is the grouped layer kernel, and every other pair raises (no
    emulation).
    """

    if weight.ndim != 2 or input.ndim < 1 or input.shape[-1] != weight.shape[0]:
        raise ValueError("native expert matmul received incompatible input/weight shapes")
    pair = (str(weight_format), str(activation_format))
    if pair not in {("mxfp8", "mxfp8"), ("nvfp4", "nvfp4")}:
        raise NativeExpertPrecisionError(
            f"no integrated native expert kernel for {weight_format}/{activation_format}; emulation is prohibited"
        )
    mm = nvfp4_mm_nt if pair[0] == "nvfp4" else mxfp8_mm_nt
    _require_cuda_bf16(input, weight, operation=f"native {pair[0].upper()} expert matmul")
    out = mm(input.reshape(-1, input.shape[-1]), weight.t())
    if bias is not None:
        out = out + bias
    return out.reshape(*input.shape[:-1], weight.shape[1])


@lru_cache(maxsize=8)
def _smoke(device_index: int, weight_format: str = "bfloat16") -> tuple[bool, str]:
    from spalmer_b200.config import MicroExpertsConfig
    from spalmer_b200.experts import B200MicroExpertChannelMixer

    try:
        device = torch.device("cuda", device_index)
        major, minor = torch.cuda.get_device_capability(device)
        if (major, minor) != (10, 0):
            return False, f"sm_{major}{minor} is not sm_100"
        config = MicroExpertsConfig(d_model=128, num_experts=16, expert_inter_dim=32, active_experts=4,
                                    shared_inter_dim=128, expert_weight_format=weight_format,
                                    expert_activation_format=weight_format)
        with torch.no_grad():
            gen = torch.Generator().manual_seed(1204)
            mixer = B200MicroExpertChannelMixer(config).to(device=device, dtype=torch.bfloat16)
            x = torch.randn(1, 256, 128, generator=gen).to(device=device, dtype=torch.bfloat16)
            out = mixer(x)
            torch.cuda.synchronize(device)
            ok = bool(torch.isfinite(out.update.float()).all()) and mixer.device_status() == 0
        return ok, f"libspx sm_100a grouped {weight_format} forward smoke " + ("passed" if ok else "failed")
    except Exception as error:  # noqa: BLE001 - report, never raise from discovery
        return False, f"libspx smoke failed: {error}"


def native_provider_capabilities(device: str | torch.device | None = None) -> list[dict[str, str | bool]]:
    resolved = torch.device(device if device is not None else ("cuda" if torch.cuda.is_available() else "cpu"))
    if resolved.type == "cuda" and resolved.index is None and torch.cuda.is_available():
        resolved = torch.device("cuda", torch.cuda.current_device())
    claims = []
    for fmt in ("bfloat16", "mxfp8", "nvfp4"):
        if resolved.type != "cuda" or not torch.cuda.is_available():
            available, detail = False, "CUDA is unavailable"
        else:
            available, detail = _smoke(resolved.index, fmt)
        claims.append(
            {
                "provider_id": PROVIDER_ID,
                "weight_format": fmt,
                "activation_format": fmt,
                "forward_available": available,
                "backward_available": available and fmt == "bfloat16",
                "grouped_available": available,
                "verified": available,
                "detail": detail,
            }
        )
    return claims
