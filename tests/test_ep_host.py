"""Expert-parallel exchange logic on CPU: the plan functions, and a
world_size-2 gloo run of `ExpertParallelMixer` (production exchange code)
with the oracle stages, which must reproduce the single-process layer
bit for bit."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spalmer_b200.ep import exchange_plan, experts_per_rank, receive_expert_ids


def test_experts_per_rank():
    assert experts_per_rank(200, 8) == 25
    assert experts_per_rank(200, 1) == 200
    with pytest.raises(ValueError):
        experts_per_rank(200, 3)


def test_exchange_plan_and_receive_ids():
    # rank 1 of 2, E = 6 (3 per rank)
    local_counts = np.array([4, 0, 1, 2, 2, 5])          # this rank's pairs per expert
    recv_counts = np.array([3, 0, 2,   2, 2, 5])         # [src0: experts 3..5, src1: experts 3..5]
    plan = exchange_plan(local_counts, recv_counts, 2)
    assert plan.send_rows == [5, 9]
    assert plan.recv_rows == [5, 9]
    ids = receive_expert_ids(plan, torch.device("cpu")).tolist()
    assert ids == [0, 0, 0, 2, 2] + [0, 0, 1, 1, 2, 2, 2, 2, 2]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


CFG = dict(d_model=64, num_experts=8, expert_inter_dim=32, shared_inter_dim=64, active_experts=2)


def _build():
    from spalmer_b200 import B200MicroExpertChannelMixer, MicroExpertsConfig
    from tests.helpers import oracle_params

    torch.manual_seed(0)
    mixer = B200MicroExpertChannelMixer(MicroExpertsConfig(**CFG)).to(torch.bfloat16)
    x = torch.randn(4, 16, 64, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    return mixer, oracle_params(mixer), x


def _worker(rank: int, world: int, port: int, out_dir: str, dedup: bool = False) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from spalmer_b200.ep import ExpertParallelMixer
        from tests.ep_oracle_ops import OracleOps

        mixer, params, x = _build()
        mine = x.chunk(world, dim=0)[rank].contiguous()
        ep = ExpertParallelMixer(mixer, ops=OracleOps(params, CFG["active_experts"], rank, world), dedup=dedup)
        out = ep(mine)
        torch.save({"update": out["update"], "send": out["send_rows"], "recv": out["recv_rows"],
                    "send_pairs": out.get("send_pairs")}, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_ep_exchange_matches_single_process_gloo(tmp_path):
    from tests.ep_oracle_ops import OracleOps, single_process_update

    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    _, params, x = _build()
    got = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    # each rank's update equals the layer run on its own tokens in one process
    for r, part in enumerate(x.chunk(world, dim=0)):
        want = single_process_update(OracleOps(params, CFG["active_experts"], 0, 1),
                                     part.reshape(-1, 64).contiguous())
        assert torch.equal(got[r]["update"].reshape(-1, 64).view(torch.int16), want.view(torch.int16))
    # every row sent was received: rank a's send to b == rank b's receive from a
    assert got[0]["send"][1] == got[1]["recv"][0] and got[1]["send"][0] == got[0]["recv"][1]
    assert sum(got[0]["send"]) == x.shape[1] * x.shape[0] // world * CFG["active_experts"]


def test_ep_dedup_exchange_matches_single_process_gloo(tmp_path):
    """Rows sent once per destination rank, pair rows summed per destination:
    the update matches the single-process layer within BF16 tolerance, and
    fewer rows travel than pairs."""

    from tests.ep_oracle_ops import OracleOps, single_process_update

    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), True), nprocs=world, join=True)
    _, params, x = _build()
    got = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    for r, part in enumerate(x.chunk(world, dim=0)):
        want = single_process_update(OracleOps(params, CFG["active_experts"], 0, 1),
                                     part.reshape(-1, 64).contiguous()).float()
        have = got[r]["update"].reshape(-1, 64).float()
        assert ((have - want).abs() <= 1e-2 + 2e-2 * want.abs()).all()
    assert got[0]["send"][1] == got[1]["recv"][0] and got[1]["send"][0] == got[0]["recv"][1]
    tokens = x.shape[0] * x.shape[1] // world
    for g in got:
        assert sum(g["send"]) <= tokens * world  # at most one row per token and destination
        assert sum(g["send_pairs"]) == tokens * CFG["active_experts"]
        assert sum(g["send"]) < sum(g["send_pairs"])
