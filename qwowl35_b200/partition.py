"""Ragged-batch partitioner: which sequences each GPU decodes.

The decode step shards by sequence.  Every rank holds a full weight replica
and owns the recurrent state and KV chunks of its sequences, so a step moves
on rank r

    weights                     (read once per step, whatever the batch)
  + sum over its sequences of   state bytes (DeltaNet state read + written)
                              + KV bytes (the sequence's whole cache, read)

and the job runs at the pace of the rank with the most bytes.  The reference
serves independent sessions (qw35-server/src/model.rs:269-304: one runtime
per session over one mapping); this module decides which sessions live on
which GPU.  There is no data-path collective.

`partition` is greedy longest-processing-time: sequences in decreasing cost
order, each to the rank with the least load so far (ties to the lowest rank).
Its makespan is within 4/3 of optimal (Graham's bound), and every rank
computes the same assignment from the same lengths, so ranks need no
exchange beyond agreeing on the batch.
"""
from __future__ import annotations

from dataclasses import dataclass

CHUNK = 256  # KV positions per chunk (QW35_KV_CHUNK)


@dataclass(frozen=True)
class StepCost:
    """Bytes one decode step moves for the Qwen3.5-9B shape (config 5)."""
    weight_bytes: int = 5_715_000_000  # GF4 FFN + Q8_0 projections/head/embedding row, read once per step
    delta_layers: int = 24
    attn_layers: int = 8
    state_bytes_per_layer: int = 2 * 32 * 128 * 128 * 4 + 2 * 8192 * 3 * 4  # SSM + conv state, read + write
    kv_bytes_per_position: int = 4 * 256 * 2 * 2  # K + V rows of 4 kv heads x 256 dims, f16 (q8_0: 4 * 272 * 2)

    def sequence(self, length: int) -> int:
        """Bytes of one sequence at `length` positions (its per-step share)."""
        return self.delta_layers * self.state_bytes_per_layer + self.attn_layers * self.kv_bytes_per_position * length


def partition(lengths: list[int], n_ranks: int, cost: StepCost | None = None) -> list[list[int]]:
    """Indices of `lengths` per rank, balancing per-step bytes (see the module doc)."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    cost = cost or StepCost()
    order = sorted(range(len(lengths)), key=lambda i: (-cost.sequence(lengths[i]), i))
    load = [0] * n_ranks
    out: list[list[int]] = [[] for _ in range(n_ranks)]
    for i in order:
        r = min(range(n_ranks), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += cost.sequence(lengths[i])
    for part in out:
        part.sort()
    return out


def rank_bytes(lengths: list[int], parts: list[list[int]], cost: StepCost | None = None) -> list[int]:
    """Per-step bytes of each rank under an assignment (weights included)."""
    cost = cost or StepCost()
    return [cost.weight_bytes + sum(cost.sequence(lengths[i]) for i in p) for p in parts]


def imbalance(lengths: list[int], parts: list[list[int]], cost: StepCost | None = None) -> float:
    """Slowest rank's bytes over the mean rank's (1.0 = perfectly balanced)."""
    b = rank_bytes(lengths, parts, cost)
    return max(b) / (sum(b) / len(b))


def log_uniform_lengths(n: int, lo: int = 512, hi: int = 131072, seed: int = 4) -> list[int]:
    """Context lengths log-uniform in [lo, hi] (BASELINE config 4's distribution), seeded."""
    import numpy as np

    rng = np.random.default_rng(seed)
    return [int(v) for v in np.exp(rng.uniform(np.log(lo), np.log(hi), n)).astype(np.int64)]
