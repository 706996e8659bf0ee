"""The bench's multi-rank host logic on CPU: two ranks over gloo (the GPU
runs use NCCL, one rank per GPU). Sequences shard across ranks with no
collective on the data path; the only exchanges are the timing's maximum
over ranks and the barriers around the timed region, and the reference arm
runs on rank 0 alone."""
import json
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # each rank's own total time; every rank must see the slowest
        own_ms = 1000.0 + 250.0 * rank
        slowest = bench.max_over_ranks(own_ms, world, torch, dist)
        dist.barrier()
        value = bench.weak_value(world, 16384 * 10, slowest)
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump({"slowest": slowest, "value": value}, f)
    finally:
        dist.destroy_process_group()


def test_two_ranks_agree_on_the_slowest_time_and_the_job_throughput(tmp_path):
    world, port = 2, _free_port()
    mp.start_processes(_rank, args=(world, port, str(tmp_path)), nprocs=world, start_method="spawn", join=True)
    got = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(world)]
    assert all(g["slowest"] == 1250.0 for g in got)
    # all ranks' tokens over the slowest rank's seconds
    assert all(g["value"] == pytest.approx(2 * 16384 * 10 / 1.25) for g in got)


def test_reference_arm_runs_on_rank_zero_only(capsys):
    sys.path.insert(0, ROOT)
    import bench
    bench.run_reference(None, 1, 2)  # rank 1 of 2: returns before any work
    assert capsys.readouterr().out == ""
