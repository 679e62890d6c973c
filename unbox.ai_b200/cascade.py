"""Shared-prefix (cascade) decode attention: radix-shared pages read once per step.

The reference's radix cache gives requests with a common prompt prefix the same
physical pages (unbox_platform/infer/kvcache.py:97-122), and
paged_decode_attention_ref (kernels/paged_decode_attention.py:157-191) then reads
those pages once per request. ``plan_cascade`` finds, once per decode step and
on the host (where the engine builds its block tables, engine.py:179-185), the
groups of requests whose block-table rows start with the same pages, and
``paged_attention_cascade`` computes

    out[b] = merge( attention of b over its own suffix pages,
                    attention of b over the group's shared pages )

with, in one launch, every request's suffix (the balanced decode kernel, KV
append fused, returning log-sum-exps) on most SMs and all groups' shared pages
on the others (each page chunk of a KV head loaded into shared memory once for
up to 128 (request, head) rows of the group, tcgen05 tensor-core MMAs with
accumulators in tensor memory), then one merge launch. Softmax splits exactly
over disjoint key sets, so the result is the attention over the whole context.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from . import library as _L
from .ops import _DTYPES, _SCHEDULES, _require_cuda, _stream, workspace_for

MAX_CHUNK_PAGES = 8     # shared pages of one tensor-core chunk (kCascadeMaxPages)
MAX_ITEM_PAGES = 64     # shared pages of one work item, taken a chunk at a time (kCascadeMaxItemPages)
TILE_ROWS = 128         # (request, head) rows one CTA covers: the M of its tensor-core tile
WORK_INTS = 6
# Cost model that splits the SMs of the one-launch step between the two passes
# (B200 measurements on the radix workload): a suffix CTA streams a page of all
# KV heads in about PAGE_US after about SUFFIX_FIXED_US of start-up and merge; a
# prefix pipeline (two per CTA, running side by side) takes a (work item, KV
# head) pair in about ITEM_US plus CHUNK_US per 8-page chunk of the item.
PAGE_US = 1.2
SUFFIX_FIXED_US = 8.0
ITEM_US = 4.0
CHUNK_US = 8.0


@dataclass
class CascadePlan:
    """Device-side description of one decode step's prefix groups (shared by all layers)."""
    suffix_block_table: torch.Tensor   # (B, max_blocks) int32: rows from the first unshared page
    suffix_context_lens: torch.Tensor  # (B,) int32: context minus the shared tokens
    page_list: torch.Tensor            # int32: shared pages of every group
    member_list: torch.Tensor          # int32: member sequences of every group
    work: torch.Tensor                 # (W, 6) int32
    merge_items: torch.Tensor          # (M, 2) int32: (sequence, prefix chunks)
    max_chunks: int                    # partial rows per (member, head): work items along the prefix
    groups: list = field(default_factory=list)   # host: (members, shared pages) per group
    shared_tokens: int = 0             # tokens the shared pages hold, once per group
    suffix_pages: int = 0              # pages of every request's suffix (host count)
    prefix_chunks: int = 0             # 8-page chunks of all work items (host count)
    _lse: Optional[torch.Tensor] = None
    _ws: Optional[torch.Tensor] = None
    _split: dict = field(default_factory=dict)  # per-plan host caches: SM split, workspace sizing

    @property
    def num_work(self) -> int:
        return int(self.work.shape[0])

    @property
    def num_merge(self) -> int:
        return int(self.merge_items.shape[0])


def plan_cascade(block_table, context_lens, num_heads: int, num_kv_heads: int, block_size: int = 16,
                 min_shared_pages: int = 4, max_parts: int = 4, device=None) -> CascadePlan:
    """Group the requests of one decode step by shared leading pages.

    A group is the requests whose rows start with the same page id; its shared
    prefix is the longest run of leading page ids all members have in common,
    cut so that every member keeps at least one token of its own (the token being
    decoded is written to a private page) and before any page that holds some
    request's append slot (the shared pages are read while the suffix pass
    appends). Groups with fewer than
    ``min_shared_pages`` shared pages, or a single member, stay on the plain path.
    The shared pages are split into at most ``max_parts`` runs of whole 8-page
    chunks (at most 64 pages each): one work item per run and block of up to
    128 / G members, one partial row per (member, head) and run.
    ``block_table`` / ``context_lens`` are host arrays (or CPU tensors).
    """
    bt = np.asarray(block_table.cpu() if isinstance(block_table, torch.Tensor) else block_table, dtype=np.int32)
    ctx = np.asarray(context_lens.cpu() if isinstance(context_lens, torch.Tensor) else context_lens,
                     dtype=np.int64)
    B, MB = bt.shape
    G = num_heads // num_kv_heads
    max_members = TILE_ROWS // G
    suffix_bt = bt.copy()
    suffix_ctx = ctx.astype(np.int32).copy()
    pages, members, work, merge, groups = [], [], [], [], []
    max_chunks = 1
    shared_tokens = 0
    # pages that receive this step's appended token (position ctx - 1)
    last = (ctx - 1) // block_size
    has_last = (ctx >= 1) & (last < MB)
    append_pages = np.unique(bt[np.nonzero(has_last)[0], last[has_last]])
    eligible = np.nonzero((ctx > block_size) & (bt[:, 0] >= 0))[0]
    firsts = bt[eligible, 0]
    for first in np.unique(firsts):
        mem = eligible[firsts == first]
        if mem.size < 2:
            continue
        rows = bt[mem]
        eq = np.all(rows == rows[0], axis=0) & (rows[0] >= 0)
        P = int(np.argmin(eq)) if not eq.all() else MB
        P = min(P, int(((ctx[mem] - 1) // block_size).min()))
        hit = np.isin(rows[0, :P], append_pages)
        if hit.any():
            P = int(np.argmax(hit))
        if P < min_shared_pages:
            continue
        # the prefix in at most max_parts runs of whole chunks (one work item
        # per run and member block; the item's chunks are folded in one after
        # another on the device, each (member, head) gets one partial per run)
        n_chunks = (P + MAX_CHUNK_PAGES - 1) // MAX_CHUNK_PAGES
        run = min(MAX_ITEM_PAGES, -(-n_chunks // max(1, max_parts)) * MAX_CHUNK_PAGES)
        n_parts = (P + run - 1) // run
        max_chunks = max(max_chunks, n_parts)
        pg_off, m_off = len(pages), len(members)
        pages.extend(int(x) for x in rows[0, :P])
        members.extend(int(b) for b in mem)
        for c in range(n_parts):
            p0 = c * run
            np_c = min(run, P - p0)
            for m0 in range(0, mem.size, max_members):
                nm = min(max_members, mem.size - m0)
                work.append((m_off + m0, nm, pg_off + p0, np_c, c, 0))
        merge.extend((int(b), n_parts) for b in mem)
        suffix_bt[mem, :MB - P] = bt[mem, P:]
        suffix_bt[mem, MB - P:] = -1
        suffix_ctx[mem] = (ctx[mem] - P * block_size).astype(np.int32)
        groups.append((mem.tolist(), rows[0, :P].tolist()))
        shared_tokens += P * block_size
    dev = torch.device(device) if device is not None else torch.device("cuda")

    def t(a, shape=None):
        arr = np.asarray(a, dtype=np.int32)
        if shape is not None:
            arr = arr.reshape(shape)
        return torch.from_numpy(np.ascontiguousarray(arr)).to(dev)

    return CascadePlan(
        suffix_block_table=t(suffix_bt), suffix_context_lens=t(suffix_ctx),
        page_list=t(pages if pages else [0]), member_list=t(members if members else [0]),
        work=t(work if work else np.zeros((0, WORK_INTS)), (-1, WORK_INTS)),
        merge_items=t(merge if merge else np.zeros((0, 2)), (-1, 2)),
        max_chunks=max_chunks, groups=groups, shared_tokens=shared_tokens,
        suffix_pages=int(((np.maximum(suffix_ctx, 0).astype(np.int64) + block_size - 1) // block_size).sum()),
        prefix_chunks=sum(-(-int(w[3]) // MAX_CHUNK_PAGES) for w in work))


def one_launch_possible(num_kv_heads: int, head_dim: int, elem_bytes: int = 2) -> bool:
    """Whether the suffix pass of these head shapes runs one balanced CTA per SM
    holding every KV head (the condition for sharing its launch with the
    shared-prefix pass): the C library's plan puts all KV heads in one CTA when a
    16-row page tile of them fits 36 KB, and one CTA per SM when that CTA has
    8 or more consumer warps (one per KV head)."""
    row = num_kv_heads * head_dim * elem_bytes
    pitch = row if (row // 16) % 2 else row + 16
    return num_kv_heads >= 8 and 16 * pitch <= 36864


def prefix_ctas_for(plan: CascadePlan, num_kv_heads: int, num_sms: int) -> int:
    """CTAs of the one-launch step that run the shared-prefix pairs: the
    smallest count (at most half the SMs) that minimises the estimated time of
    the slower pass -- the pairs go round-robin to two pipelines per CTA, the
    suffix pages are shared evenly by the other CTAs. 0 when there is no
    prefix work."""
    if plan.num_work == 0 or num_sms < 2:
        return 0
    pairs = plan.num_work * num_kv_heads
    pair_us = ITEM_US + CHUNK_US * plan.prefix_chunks / plan.num_work
    best, best_t = 1, float("inf")
    for n in range(1, num_sms // 2 + 1):
        t = max(-(-pairs // (2 * n)) * pair_us, plan.suffix_pages * PAGE_US / (num_sms - n) + SUFFIX_FIXED_US)
        if t < best_t - 1e-9:
            best, best_t = n, t
    return best


def paged_attention_cascade(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, plan: CascadePlan,
                            scale: Optional[float] = None, *, k_new: Optional[torch.Tensor] = None,
                            v_new: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                            schedule: str = "auto", overlap_previous: bool = False,
                            prefix_ctas: Optional[int] = None) -> torch.Tensor:
    """Paged decode attention (with the KV append when k_new/v_new are given) using
    ``plan``: same result as ``paged_attention`` over the original block tables.
    The suffix and shared-prefix passes share one launch (``prefix_ctas`` CTAs
    for the prefix pairs, default from the plan's cost model; 0 runs them as two
    launches), then a merge launch. bf16/f16."""
    dev = _require_cuda(q, k_cache, v_cache)
    if q.dtype not in (torch.bfloat16, torch.float16) or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise TypeError("the cascade path is built for bf16/f16 (use paged_attention for fp32)")
    if (k_new is None) != (v_new is None):
        raise ValueError("pass both k_new and v_new, or neither")
    B, H, D = q.shape
    NB, bs, KVH, D2 = k_cache.shape
    if D2 != D or k_cache.stride() != v_cache.stride() or q.stride(-1) != 1 or k_cache.stride(-1) != 1:
        raise ValueError("q (B, H, D) and caches (NB, bs, KVH, D) with contiguous last dimensions expected")
    sbt, sctx = plan.suffix_block_table, plan.suffix_context_lens
    if sbt.shape[0] != B or sctx.shape != (B,):
        raise ValueError("the plan was made for another batch")
    if out is None:
        out = torch.empty((B, H, D), dtype=q.dtype, device=dev)
    elif out.shape != (B, H, D) or out.dtype != q.dtype or out.stride(-1) != 1:
        raise ValueError("out must be (B, H, D) in q's dtype with a contiguous last dimension")
    if B == 0:
        return out
    if scale is None:
        scale = D ** -0.5
    lib = _L.load()
    if plan._lse is None or plan._lse.shape != (B, H) or plan._lse.device != dev:
        plan._lse = torch.empty((B, H), dtype=torch.float32, device=dev)
    if plan._ws is None or plan._ws.device != dev or plan._split.get("ws") != (B, H, D):
        need = ctypes.c_size_t(0)
        _L.check(lib.ubx_cascade_workspace_size(B, H, D, plan.max_chunks, ctypes.byref(need)), "cascade workspace")
        if plan._ws is None or plan._ws.numel() < need.value or plan._ws.device != dev:
            plan._ws = torch.empty(max(int(need.value), 256), dtype=torch.uint8, device=dev)
        plan._split["ws"] = (B, H, D)
    dws = workspace_for(dev)
    buf = dws.ensure(B, H, D, sbt.shape[1], 0, KVH, q.dtype)
    if prefix_ctas is None:
        key = (KVH, dws.num_sms)
        if key not in plan._split:
            plan._split[key] = prefix_ctas_for(plan, KVH, dws.num_sms)
        prefix_ctas = plan._split[key]
    if k_new is not None:
        _require_cuda(q, k_new, v_new)
        if k_new.shape != (B, KVH, D) or v_new.shape != k_new.shape or k_new.dtype != q.dtype or \
                v_new.dtype != q.dtype or k_new.stride() != v_new.stride() or k_new.stride(-1) != 1:
            raise ValueError(f"k_new / v_new must be ({B}, {KVH}, {D}) in q's dtype with equal strides")
        kn, vn, ns0, ns1 = k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), k_new.stride(1)
    else:
        kn, vn, ns0, ns1 = None, None, 0, 0
    st = lib.ubx_cascade_attention(
        kn, vn, ns0, ns1, q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(),
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), sbt.data_ptr(), sbt.stride(0), sctx.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1), B, H, KVH, D, bs, NB, sbt.shape[1], float(scale),
        _DTYPES[q.dtype], _SCHEDULES[schedule], plan.page_list.data_ptr(), plan.member_list.data_ptr(),
        plan.work.data_ptr(), plan.num_work, plan.merge_items.data_ptr(), plan.num_merge, plan.max_chunks,
        int(prefix_ctas), _L.FLAG_OVERLAP_PREVIOUS if overlap_previous else 0, plan._lse.data_ptr(),
        buf.data_ptr(), buf.numel(), plan._ws.data_ptr(), plan._ws.numel(), _stream(dev))
    _L.check(st, "cascade attention")
    return out
