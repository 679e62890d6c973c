"""Partitioning a decode batch across GPUs (one process per GPU, no collective).

Decode attention is independent per (sequence, KV head), so a box of GPUs
splits the work without exchanging anything on the data path. This mirrors
how the reference spreads requests over one worker per GPU
(unbox_platform/infer/router.py:85-86 round-robins requests over workers;
unbox_platform/infer/worker.py:47-51 pins one worker per GPU), with two
refinements for a fixed batch:

* requests are placed by greedy LPT on their KV bytes (longest first onto the
  least-loaded GPU), so GPU loads differ by at most one request;
* requests longer than ``long_threshold`` tokens are split by KV head: every
  GPU holds ``num_kv_heads / world`` KV heads (and their query heads) of each
  such request, so one very long context cannot dominate a single GPU.

``plan_shards`` is pure host logic (numpy); ``local_layout`` builds the
per-rank paging metadata (its own page pool, permuted per rank).
"""
from __future__ import annotations

import dataclasses
import heapq
from typing import List, Optional

import numpy as np


@dataclasses.dataclass
class RankShard:
    rank: int
    whole: np.ndarray            # sequence indices attended in full on this rank (ascending)
    head_split: np.ndarray       # long sequences of which this rank holds a KV-head slice
    kv_head_first: int           # first KV head of the slice
    kv_head_count: int           # KV heads in the slice (0 when head_split is empty)
    kv_bytes: int                # K+V bytes this rank streams per layer


def lpt(costs: np.ndarray, bins: int, start: Optional[np.ndarray] = None) -> List[List[int]]:
    """Greedy longest-processing-time assignment of items to `bins` bins.

    Items are taken in decreasing cost (ties by index) and each goes to the bin
    with the smallest load so far (ties by bin index). Returns the item indices
    of every bin, ascending.
    """
    load = [(float(start[i]) if start is not None else 0.0, i) for i in range(bins)]
    heapq.heapify(load)
    out: List[List[int]] = [[] for _ in range(bins)]
    order = sorted(range(len(costs)), key=lambda i: (-float(costs[i]), i))
    for i in order:
        l, b = heapq.heappop(load)
        out[b].append(i)
        heapq.heappush(load, (l + float(costs[i]), b))
    return [sorted(x) for x in out]


def plan_shards(context_lens: np.ndarray, world: int, num_kv_heads: int = 8, head_dim: int = 112,
                elem_bytes: int = 2, long_threshold: int = 2048) -> List[RankShard]:
    """Split a decode batch over `world` GPUs (see module docstring)."""
    ctx = np.asarray(context_lens, dtype=np.int64)
    row = 2 * head_dim * elem_bytes  # K + V bytes of one token of one KV head
    split_heads = world > 1 and num_kv_heads % world == 0
    long = (ctx > long_threshold) if split_heads else np.zeros_like(ctx, dtype=bool)
    long_idx = np.nonzero(long)[0]
    short_idx = np.nonzero(~long)[0]
    per = num_kv_heads // world if split_heads else num_kv_heads
    head_load = float(ctx[long_idx].sum()) * per * row
    bins = lpt(ctx[short_idx] * num_kv_heads * row, world, start=np.full(world, head_load))
    shards = []
    for r in range(world):
        whole = short_idx[bins[r]] if len(bins[r]) else np.zeros(0, dtype=np.int64)
        kvb = int(ctx[whole].sum() * num_kv_heads * row + head_load)
        shards.append(RankShard(r, np.asarray(whole, dtype=np.int64), long_idx.copy(),
                                r * per if len(long_idx) else 0, per if len(long_idx) else 0, kvb))
    return shards


def check_cover(shards: List[RankShard], batch: int, num_kv_heads: int) -> None:
    """Every (sequence, KV head) pair is owned by exactly one rank."""
    own = np.zeros((batch, num_kv_heads), dtype=np.int64)
    for s in shards:
        own[s.whole, :] += 1
        if s.kv_head_count:
            own[np.ix_(s.head_split, np.arange(s.kv_head_first, s.kv_head_first + s.kv_head_count))] += 1
    if not np.all(own == 1):
        raise AssertionError("shards do not cover every (sequence, KV head) exactly once")


def local_layout(context_lens: np.ndarray, seqs: np.ndarray, seed: int, num_heads: int, num_kv_heads: int,
                 head_dim: int = 112, block_size: int = 16):
    """Paging metadata of one rank's share: its own pool, pages permuted per rank."""
    from .workloads import Layout, _assign_pages, portable_permutation
    ctx = np.asarray(context_lens, dtype=np.int64)[seqs].astype(np.int32)
    if ctx.size == 0:
        return None
    need = int(((ctx.astype(np.int64) + block_size - 1) // block_size).sum())
    perm = portable_permutation(seed, 2, need)
    bt, _ = _assign_pages(ctx.astype(np.int64), perm, block_size)
    return Layout(ctx, bt, need, num_heads, num_kv_heads, head_dim, block_size)
