"""Expert parallelism on 2 GPUs over NCCL: every rank's update (and routing)
equals the single-GPU layer on the same tokens, bit for bit, for BF16 and
mixed BF16/MXFP8 experts.  Skipped with fewer than 2 GPUs."""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CFG = dict(d_model=256, num_experts=200, expert_inter_dim=64, shared_inter_dim=256, active_experts=8)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mxfp8: bool, out_dir: str, dedup: bool = False,
            exchange: str | None = None, peer_rows: str = "store") -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=device)
    try:
        from spalmer_b200 import B200MicroExpertChannelMixer
        from spalmer_b200.ep import ExpertParallelMixer
        from tests.helpers import mxfp8_config, mxfp8_experts, set_mxfp8_lanes
        from spalmer_b200 import MicroExpertsConfig

        config = mxfp8_config(**CFG) if mxfp8 else MicroExpertsConfig(**CFG)
        torch.manual_seed(0)
        mixer = B200MicroExpertChannelMixer(config).to(torch.bfloat16).eval().to(device)
        if mxfp8:
            set_mxfp8_lanes(mixer, mxfp8_experts(config.num_experts, 0.25))
        x = torch.randn(8, 512, CFG["d_model"], generator=torch.Generator().manual_seed(1 + rank))
        x = x.to(torch.bfloat16).to(device)
        ep = ExpertParallelMixer(mixer, dedup=dedup, exchange=exchange, peer_rows=peer_rows)
        with torch.no_grad():
            first = ep(x)
            got = ep(x)  # buffers reused
            want = mixer(x)
        torch.cuda.synchronize()
        ep.close()
        res = {
            "update_equal": torch.equal(got["update"], want.update),
            "ids_equal": torch.equal(got["expert_ids"], want.metrics["expert_ids"]),
            "weights_equal": torch.equal(got["routing_weights"], want.metrics["routing_weights"]),
            "max_diff": float((got["update"].float() - want.update.float()).abs().max()),
            "within_tol": bool(((got["update"].float() - want.update.float()).abs()
                                <= 1e-2 + 2e-2 * want.update.float().abs()).all()),
            "repeat_equal": torch.equal(first["update"], got["update"]),
            "send": got["send_rows"], "recv": got["recv_rows"], "status": mixer.device_status(),
        }
        torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["peer", "peer_load", "nccl"])
@pytest.mark.parametrize("mxfp8", [False, True])
def test_expert_parallel_matches_single_gpu(tmp_path, mxfp8, exchange):
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    peer_rows = "load" if exchange == "peer_load" else "store"
    exchange = "peer" if exchange == "peer_load" else exchange
    mp.spawn(_worker, args=(world, _free_port(), mxfp8, str(tmp_path), False, exchange, peer_rows), nprocs=world,
             join=True)
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    for r in res:
        assert r["status"] == 0
        assert r["ids_equal"] and r["weights_equal"]
        assert r["update_equal"], r["max_diff"]
        assert r["repeat_equal"]
    assert res[0]["send"][1] == res[1]["recv"][0] and res[1]["send"][0] == res[0]["recv"][1]
    assert np.sum(res[0]["send"]) == 8 * 512 * CFG["active_experts"]


@pytest.mark.parametrize("mxfp8", [False, True])
def test_expert_parallel_dedup_matches_single_gpu(tmp_path, mxfp8):
    """Rows once per destination GPU: routing identical, update within BF16 tolerance."""

    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_worker, args=(world, _free_port(), mxfp8, str(tmp_path), True), nprocs=world, join=True)
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    for r in res:
        assert r["status"] == 0
        assert r["ids_equal"] and r["weights_equal"]
        assert r["within_tol"], r["max_diff"]
    assert res[0]["send"][1] == res[1]["recv"][0] and res[1]["send"][0] == res[0]["recv"][1]
    assert sum(res[0]["send"]) < 8 * 512 * CFG["active_experts"]
