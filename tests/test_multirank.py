"""Host-side logic of the multi-GPU bench on CPU: two gloo ranks.

The decode step shards by sequence (each rank owns its sequences, weights are
replicated, no data-path collective); the only cross-rank operations are the
barriers around the timed region and the MAX reduction of the per-rank
device times, which these tests run with the gloo backend.
"""
import os
import socket
import subprocess
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r, w, local = bench.dist_env()
        assert (r, w, local) == (rank, world, rank)
        dist.barrier()
        # per-rank device times: the job takes as long as its slowest rank
        slowest = bench.max_over_ranks(1.0 + 0.5 * rank, world, torch.device("cpu"))
        args = SimpleNamespace(batch=32, ctx_fill=4096, layers=32)
        cfg = bench.workload_config(args, world)
        out.put((rank, slowest, cfg["global_batch"], cfg["parallelism"]))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_the_slowest_time_and_the_global_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    assert [g[1] for g in got] == [1.5, 1.5]           # MAX over ranks
    assert all(g[2] == 64 for g in got)                 # 32 sequences per GPU, weak scaling
    assert all(g[3].startswith("dp2") for g in got)


def test_single_rank_reduction_is_the_identity():
    assert bench.max_over_ranks(0.25, 1, torch.device("cpu")) == 0.25


def test_reference_arm_rank_one_exits_without_work():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1", MASTER_ADDR="127.0.0.1")
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "3"], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""  # only rank 0 prints the reference line


@pytest.mark.parametrize("env,expect", [({}, (0, 1, 0)), ({"RANK": "3", "WORLD_SIZE": "8", "LOCAL_RANK": "3"}, (3, 8, 3))])
def test_dist_env_reads_torchrun_variables(monkeypatch, env, expect):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    assert bench.dist_env() == expect
