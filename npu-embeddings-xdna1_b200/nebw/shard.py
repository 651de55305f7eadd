"""Data-parallel sharding of one request batch over GPUs, and the gather.

Every sequence is an independent encoder pass (the reference computes rows
independently: gemm_nt, LayerNorm and pooling are row-local and attention is
per (sequence, head) -- runtime/include/common/conv_host.hpp:154-158,
runtime/src/encoders/bert_encoder.cpp:1001-1004), so a batch splits across
ranks with one weight replica per GPU and no collective on the data path.
The only exchange is the end of the step: the [B, hidden] fp32 embeddings
are gathered to the serving rank and put back in request order.

plan_shards is deterministic and needs no communication: every rank computes
the same plan from the same lengths.
"""

from __future__ import annotations

import numpy as np


def shard_cost(lens) -> np.ndarray:
    """Relative cost of each sequence: linear (GEMM) plus quadratic
    (attention) in its length, in the proportion of a BERT-large layer."""
    lens = np.asarray(lens, np.float64)
    return lens + lens ** 2 / 2048.0


def plan_shards(lens, n: int) -> list[np.ndarray]:
    """Length-balanced plan: sequences in decreasing cost order, each to the
    rank with the least cost so far (ties to the lowest rank).  Returns n
    ascending index arrays that partition range(len(lens))."""
    lens = np.asarray(lens)
    if n < 1:
        raise ValueError("need at least one rank")
    if n == 1:
        return [np.arange(len(lens))]
    cost = shard_cost(lens)
    order = np.argsort(-cost, kind="stable")
    load = np.zeros(n)
    owner = np.empty(len(lens), np.int64)
    for i in order:
        r = int(np.argmin(load))
        owner[i] = r
        load[r] += cost[i]
    return [np.nonzero(owner == r)[0] for r in range(n)]


def unpermute(gathered: np.ndarray, shards, max_b: int) -> np.ndarray:
    """[n * max_b, H] rank-major gathered rows -> [B, H] in request order."""
    B = sum(len(s) for s in shards)
    out = np.empty((B, gathered.shape[1]), gathered.dtype)
    for r, idx in enumerate(shards):
        out[idx] = gathered[r * max_b:r * max_b + len(idx)]
    return out


def gather_to_root(local, gather_buf, world: int, rank: int, dist, root: int = 0):
    """Gather every rank's [max_b, H] block into root's [world * max_b, H]
    buffer (torch tensors on the process group's device).  Collective: all
    ranks call it in the same order."""
    chunks = list(gather_buf.chunk(world)) if rank == root else None
    dist.gather(local, chunks, dst=root)
