"""bench.py's multi-GPU host logic with two gloo ranks on the CPU: each rank is
an independent replica; the job's time is the slowest rank's and its tokens
the sum over ranks."""
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


def _rank(rank, world, port, out):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    ms, tokens = (10.0 + rank * 2.5), 100 + rank
    out[rank] = bench.combine_ranks(dist, ms, tokens, "cpu")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_combine_ranks_gloo_world_2():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(90)
            assert p.exitcode == 0
        assert out[0] == out[1] == (12.5, 201)


def test_replica_config_names_the_parallelism():
    sys.path.insert(0, ROOT)
    import argparse

    import bench
    args = argparse.Namespace(workload="qwen2.5-1.5b", steps=8, warmup=3)
    assert bench.workload_config(args, 2)["parallelism"] == "replicas x2"
    assert bench.workload_config(args, 1)["parallelism"] == "single"
