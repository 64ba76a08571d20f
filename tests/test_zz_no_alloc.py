"""spx_dispatch_static: the dispatch sort for callers that cannot allocate.

Some callers cannot allocate device memory (an FFI client that only holds the
buffers it was handed, or code where cudaMalloc is forbidden or would
synchronise, such as global-mode stream capture).  spx_dispatch_static gives
them the same permutation and counts as spx_dispatch while keeping its scratch
in a fixed file-scope device array.  This test calls it through the C ABI twice
in a row (different shapes, so stale scratch from the first call would show),
then on the single-CTA path and at its stated limits, and compares each
result with the workspace-based entry point; the outputs are integers, so the
comparison is exact.  The status word the kernels leave in the scratch is read
back through spx_dispatch_static_status.  It runs last in the suite (file
name) and also passes on its own in a fresh process.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from spalmer_b200 import _lib, dispatch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _ids(tokens, k, experts, seed):
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, experts + 1) ** 1.1
    p /= p.sum()
    ids = np.stack([rng.choice(experts, size=k, replace=False, p=p) for _ in range(tokens)])
    return torch.from_numpy(ids.astype(np.int64)).to(DEV)


def _dims(tokens, k, experts):
    return _lib.LayerDims(tokens=tokens, d_model=64, num_experts=experts, inter_dim=16, shared_dim=0,
                          top_k=k, score_transform=1, execution_loop=0)


def _static_dispatch(ids, experts):
    lib = _lib.load()
    tokens, k = ids.shape
    order = torch.full((tokens * k,), -1, dtype=torch.int32, device=DEV)
    counts = torch.full((experts,), -1, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = lib.spx_dispatch_static(_dims(tokens, k, experts), ids.data_ptr(), order.data_ptr(),
                                 counts.data_ptr(), stream)
    _lib.check(rc, "spx_dispatch_static")
    return order, counts


def _status(clear=True) -> int:
    lib = _lib.load()
    value = _lib.ctypes.c_int(-1)
    _lib.check(lib.spx_dispatch_static_status(value, int(clear), torch.cuda.current_stream(DEV).cuda_stream),
               "spx_dispatch_static_status")
    return value.value


def test_static_scratch_dispatch_matches_workspace_dispatch_twice():
    # multi-CTA path (> 4096 pairs) twice, then the single-CTA path (<= 4096 pairs)
    for tokens, k, experts, seed in ((8192, 8, 200, 11), (1500, 4, 64, 12), (300, 4, 64, 13)):
        ids = _ids(tokens, k, experts, seed)
        want_order, want_counts = dispatch(ids, experts)
        got_order, got_counts = _static_dispatch(ids, experts)
        torch.cuda.synchronize()
        assert torch.equal(got_order, want_order)
        assert torch.equal(got_counts, want_counts)
        assert _status() == 0


def test_static_scratch_dispatch_at_its_limits():
    """Exactly 1,048,576 pairs over exactly 1,024 experts (the stated maximum)."""

    tokens, k, experts = 131072, 8, 1024
    gen = torch.Generator(device=DEV).manual_seed(14)
    ids = torch.argsort(torch.rand(tokens, experts, device=DEV, generator=gen), dim=1)[:, :k].contiguous()
    ids[:4096] = torch.arange(k, device=DEV)  # one expert far above the mean
    want_order, want_counts = dispatch(ids, experts)
    got_order, got_counts = _static_dispatch(ids, experts)
    torch.cuda.synchronize()
    assert torch.equal(got_order, want_order)
    assert torch.equal(got_counts, want_counts)
    assert _status() == 0


def test_static_scratch_dispatch_reports_bad_expert_ids():
    ids = _ids(512, 4, 64, 15)
    ids[7, 2] = 64  # outside [0, num_experts): skipped by the kernels and reported
    _static_dispatch(ids, 64)
    assert _status(clear=False) != 0
    assert _status(clear=True) != 0
    assert _status() == 0  # cleared
    good = _ids(512, 4, 64, 16)
    want_order, _ = dispatch(good, 64)
    got_order, _ = _static_dispatch(good, 64)
    assert torch.equal(got_order, want_order) and _status() == 0


def test_static_scratch_dispatch_rejects_oversized_problems():
    lib = _lib.load()
    ids = torch.zeros(1, 1, dtype=torch.int64, device=DEV)
    out = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    too_many_pairs = _dims((1 << 20) + 1, 1, 8)
    assert lib.spx_dispatch_static(too_many_pairs, ids.data_ptr(), out.data_ptr(), out.data_ptr(), stream) == -9
    too_many_experts = _dims(16, 1, 1025)
    assert lib.spx_dispatch_static(too_many_experts, ids.data_ptr(), out.data_ptr(), out.data_ptr(), stream) == -9
