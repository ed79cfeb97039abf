"""Ragged-batch partitioner (host logic of the multi-GPU decode, CPU only)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qwowl35_b200.partition import StepCost, imbalance, log_uniform_lengths, partition, rank_bytes


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_every_sequence_lands_on_exactly_one_rank(n):
    lens = log_uniform_lengths(32 * n, seed=n)
    parts = partition(lens, n)
    assert len(parts) == n
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(len(lens)))


@pytest.mark.parametrize("n", [2, 4, 8])
def test_config4_ragged_batch_is_balanced_by_step_bytes(n):
    # 32 sequences per GPU, lengths log-uniform in 512..131072
    lens = log_uniform_lengths(32 * n, seed=4)
    parts = partition(lens, n)
    assert imbalance(lens, parts) < 1.03
    # a contiguous split of the same list is what the partitioner improves on
    naive = [list(range(r * 32, (r + 1) * 32)) for r in range(n)]
    assert imbalance(lens, parts) <= imbalance(lens, naive)


def test_one_huge_sequence_goes_alone():
    lens = [131072] + [512] * 15
    parts = partition(lens, 2)
    big = next(p for p in parts if 0 in p)
    assert big == [0]  # its cache alone outweighs the fifteen short ones
    b = rank_bytes(lens, parts)
    assert max(b) == rank_bytes(lens, [[0]])[0]


def test_cost_model_counts_state_and_kv():
    c = StepCost()
    assert c.sequence(0) == 24 * (2 * 32 * 128 * 128 * 4 + 2 * 8192 * 3 * 4)
    assert c.sequence(1000) - c.sequence(0) == 8 * 4096 * 1000


def test_empty_and_invalid_inputs():
    assert partition([], 3) == [[], [], []]
    with pytest.raises(ValueError):
        partition([1, 2], 0)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lens = log_uniform_lengths(32 * world, seed=7)
        mine = partition(lens, world)[rank]
        # every rank computes the assignment alone; gather them to check they agree
        got = [None] * world
        dist.all_gather_object(got, mine)
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_compute_disjoint_covering_assignments():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res[0] == res[1]
    a, b = res[0]
    assert not set(a) & set(b) and sorted(a + b) == list(range(64))
