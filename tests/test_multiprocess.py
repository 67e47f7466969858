"""Host logic of the data-parallel path with world_size 2 over gloo on the CPU: the NCCL id that
every rank's trainer joins with is shared over the process group (ngp_b200.share_nccl_id), and the
bench's timing takes the maximum over ranks.  The GPU side (one NCCL all-reduce of the fp32
gradient per step) runs in bench.py --gpus N."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    sys.path[:0] = [str(ROOT), str(ROOT / "instant-ngp_b200")]
    import torch.distributed as dist

    import bench
    import ngp_b200

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        uid = ngp_b200.share_nccl_id()
        worst = bench.max_over_ranks(float(rank + 1) * 1.5, world)
        bench.barrier(world)
        Path(out_dir, f"rank{rank}").write_text(f"{uid.hex()} {worst}")
    finally:
        dist.destroy_process_group()


def test_two_ranks_share_nccl_id_and_max_time(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [Path(tmp_path, f"rank{r}").read_text().split() for r in range(world)]
    assert res[0][0] == res[1][0]                       # the same id on every rank
    assert bytes.fromhex(res[0][0]) != bytes(128)       # rank 0 really created one
    assert all(float(r[1]) == 3.0 for r in res)        # max over ranks


def _health_worker(rank: int, world: int, port: int, out_dir: str, mode: str) -> None:
    """Ranks step a fake training loop guarded by RankHealth; rank 1 leaves (or stops without
    leaving) after step 2, between steps; rank 0 must learn of it before its step 3."""
    sys.path[:0] = [str(ROOT), str(ROOT / "instant-ngp_b200")]
    import torch.distributed as dist

    import ngp_b200

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    health = ngp_b200.RankHealth(timeout_s=2.0, prefix=f"health_{mode}")
    dist.barrier()  # both processes are up (imports can take seconds) before the timed waits
    outcome = "finished"
    try:
        for step in range(6):
            if rank == 1 and step == 3:
                if mode == "leave":
                    health.leave()
                    outcome = "left"
                    break
                Path(out_dir, "rank1").write_text("stopped")
                os._exit(0)  # stops without telling anyone
            health.before_step(step)
    except RuntimeError as e:
        outcome = f"error: {e}"
    Path(out_dir, f"rank{rank}").write_text(outcome)
    if rank == 0:
        import time

        time.sleep(0.5)  # the store lives in rank 0: keep it up while rank 1 finishes


@pytest.mark.parametrize("mode", ["leave", "stop"])
def test_rank_health_reports_a_rank_that_left(tmp_path, mode):
    import time

    import torch.multiprocessing as mp

    t0 = time.time()
    mp.spawn(_health_worker, args=(2, _free_port(), str(tmp_path), mode), nprocs=2, join=True)
    r0 = Path(tmp_path, "rank0").read_text()
    if mode == "leave":
        assert Path(tmp_path, "rank1").read_text() == "left"
        assert r0 == "error: rank 1 left the data-parallel job before step 3"
    else:
        assert Path(tmp_path, "rank1").read_text() == "stopped"
        assert r0.startswith("error: ranks [1] did not reach step 3")
    assert time.time() - t0 < 30
