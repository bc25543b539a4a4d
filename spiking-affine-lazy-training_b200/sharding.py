"""Data-parallel sample sharding across ranks (one process per GPU).

Samples are independent (the reference vmaps the network over the batch,
salt_core/network.py:179-183), so a batch is split into per-rank shards with no data-path
collective; the only exchange is the gather of the int32 logits (the last layer's v_final) back
into the caller's sample order.

Event counts per sample vary widely (configuration 3: log-uniform 2000-20000), and a layer's cost
grows with them, so shards are balanced by events rather than by sample count: samples are taken
in decreasing event count and each goes to the rank with the fewest events so far (greedy
longest-processing-time).  The permutation is kept so the gathered logits return in input order.
"""
from __future__ import annotations

from typing import NamedTuple

import numpy as np


class Shards(NamedTuple):
    """Per-rank sample indices into the global batch; every rank holds the same number of
    slots (shorter shards are padded with `pad_index` entries whose results are dropped)."""
    index: np.ndarray      # (world, per_rank) int64 global sample index, pad_index for padding
    counts: np.ndarray     # (world,) real samples per rank
    events: np.ndarray     # (world,) events per rank
    pad_index: int

    @property
    def per_rank(self) -> int:
        return int(self.index.shape[1])

    def of(self, rank: int) -> np.ndarray:
        """The global indices rank `rank` processes, padding included."""
        return self.index[rank]


def balanced_shards(n_events: np.ndarray, world: int) -> Shards:
    """Splits samples with the given event counts over `world` ranks, balancing events."""
    n = np.asarray(n_events, dtype=np.int64).reshape(-1)
    if world < 1:
        raise ValueError("world must be >= 1")
    B = n.shape[0]
    per = max(1, -(-B // world))
    order = np.argsort(-n, kind="stable")
    load = np.zeros(world, np.int64)
    cnt = np.zeros(world, np.int64)
    slots = [[] for _ in range(world)]
    for i in order:
        open_ranks = np.nonzero(cnt < per)[0]
        r = open_ranks[np.argmin(load[open_ranks])]
        slots[r].append(int(i))
        load[r] += n[i]
        cnt[r] += 1
    index = np.full((world, per), B, np.int64)   # B = padding (dropped)
    for r in range(world):
        s = sorted(slots[r])  # keep input order inside a shard
        index[r, :len(s)] = s
    return Shards(index, cnt, load, B)


def take_shard(arrays, shards: Shards, rank: int, pad_like: int = 0):
    """Rows of each (B, ...) array for `rank`'s shard; padding slots copy row `pad_like` (any
    valid sample) with its event count set to zero by the caller where needed."""
    idx = shards.of(rank)
    safe = np.where(idx == shards.pad_index, pad_like, idx)
    return [np.ascontiguousarray(np.asarray(a)[safe]) for a in arrays]


def unshard(gathered: np.ndarray, shards: Shards) -> np.ndarray:
    """(world * per_rank, ...) rows in rank-major order -> (B, ...) rows in input order."""
    g = np.asarray(gathered)
    flat = shards.index.reshape(-1)
    keep = flat != shards.pad_index
    out = np.empty((shards.pad_index,) + g.shape[1:], dtype=g.dtype)
    out[flat[keep]] = g[keep]
    return out


def gather_rows(local, comm):
    """All-gather equally shaped (per_rank, ...) rows from every rank into (world * per_rank,
    ...) in rank order.  `comm` provides ``world`` and ``all_gather(send, recv)``: an
    ``comm.NcclComm`` for device arrays (the all-gather is then enqueued on the current stream;
    ``comm.wait()`` bounds the wait), or any object with the same two members for host arrays."""
    shape = (comm.world * local.shape[0],) + tuple(local.shape[1:])
    if isinstance(local, np.ndarray):
        out = np.empty(shape, local.dtype)
    else:
        from .device import DeviceArray
        out = DeviceArray.empty(shape, local.dtype)
    comm.all_gather(local, out)
    return out
