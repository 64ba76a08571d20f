"""The device tie-order replay (spalmer_b200/csrc/topk_exact.cuh), compiled for
the host with g++, against std::nth_element / std::partial_sort / std::sort --
the algorithms PyTorch's CPU top-k runs for the reference's routing."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ unavailable")
def test_exact_topk_replay_matches_std_algorithms(tmp_path):
    exe = tmp_path / "topk_exact_check"
    subprocess.run(
        ["g++", "-O2", "-std=c++17", str(ROOT / "tests" / "cpp" / "topk_exact_check.cpp"), "-o", str(exe)],
        check=True,
    )
    # 21 row lengths x k in 1..min(n,20) x 3000 rows, two seeds.
    for seed in (7, 8):
        out = subprocess.run([str(exe), "3000", str(seed)], capture_output=True, text=True, timeout=600)
        assert out.returncode == 0, out.stdout + out.stderr
        assert out.stdout.startswith("OK"), out.stdout
