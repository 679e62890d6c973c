"""Torch-facing host API over the C ABI (device memory and streams come from torch).

Mirrors the reference's operator interface for this path:

* ``paged_decode_attention(q, k_pool, v_pool, block_tables, seq_lens, block_size)``
  -- same name, arguments, shapes and return as
  unbox_platform/infer/kernels/paged_decode_attention.py:106-150 (and the CPU
  path at :157-191): out (B, H, D) in q's dtype, scale = head_dim ** -0.5.
* ``paged_attention(q, k_cache, v_cache, block_table, context_lens, scale)``
  -- the same op with the scale passed in.
* ``kv_append(k_new, v_new, k_cache, v_cache, slot_mapping)`` -- one launch in
  place of the per-sequence ``PagedKVCache.write_kv`` loop
  (unbox_platform/infer/engine.py:213-215, kvcache.py:330-340).
* ``slot_mapping(block_table, positions, block_size)`` -- kvcache.py:338-339 on
  the device.

Every op launches on torch's current CUDA stream, never synchronises, and
raises if the CUDA library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import library as _L

_DTYPES = {torch.float32: _L.DTYPE_F32, torch.bfloat16: _L.DTYPE_BF16, torch.float16: _L.DTYPE_F16}
_SCHEDULES = {"auto": _L.SCHEDULE_AUTO, "balanced": _L.SCHEDULE_BALANCED, "split": _L.SCHEDULE_SPLIT}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts):
    dev = ts[0].device
    for t in ts:
        if t.device.type != "cuda":
            raise ValueError("unbox_b200 ops run on CUDA tensors only (no CPU fallback)")
        if t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


class DecodeWorkspace:
    """Device workspace of the attention op: partial results of split sequences,
    merge counters and the device error word.

    One per device by default (``workspace_for``). It is zeroed when allocated and
    grows (re-allocated, zeroed) when a call needs more. Allocate it (e.g. by a
    warm-up call) before capturing a CUDA graph.
    """

    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        self.buf: Optional[torch.Tensor] = None

    @property
    def nbytes(self) -> int:
        return 0 if self.buf is None else self.buf.numel()

    def ensure(self, batch: int, num_heads: int, head_dim: int, max_blocks: int, split_pages: int = 0):
        lib = _L.load()
        need = ctypes.c_size_t(0)
        with torch.cuda.device(self.device):
            _L.check(lib.ubx_paged_decode_workspace_size(batch, num_heads, head_dim, max_blocks, split_pages,
                                                         ctypes.byref(need)), "workspace size")
        n = max(int(need.value), 1 << 20)
        if self.buf is None or self.buf.numel() < n:
            self.buf = torch.zeros(n, dtype=torch.uint8, device=self.device)
            _L.check(lib.ubx_workspace_init(self.buf.data_ptr(), self.buf.numel(), _stream(self.device)),
                     "workspace init")
        return self.buf

    def error_word_ptr(self) -> int:
        if self.buf is None:
            self.ensure(1, 1, 64, 1)
        return self.buf.data_ptr()

    def read_errors(self, clear: bool = True) -> int:
        if self.buf is None:
            return 0
        lib = _L.load()
        v = ctypes.c_int32(0)
        _L.check(lib.ubx_read_device_error(self.buf.data_ptr(), ctypes.byref(v), int(clear), _stream(self.device)),
                 "read device error")
        return int(v.value)

    def reset(self):
        """Re-zero the merge counters and the error word (after a device error)."""
        if self.buf is not None:
            _L.check(_L.load().ubx_workspace_init(self.buf.data_ptr(), self.buf.numel(), _stream(self.device)),
                     "workspace init")


_workspaces: dict = {}


def workspace_for(device: torch.device) -> DecodeWorkspace:
    key = torch.device(device).index if torch.device(device).index is not None else torch.cuda.current_device()
    ws = _workspaces.get(key)
    if ws is None:
        ws = _workspaces[key] = DecodeWorkspace(torch.device("cuda", key))
    return ws


def check_device_errors(device=None):
    """Raise if any op on ``device`` (default: all used devices) flagged bad data.

    Synchronises the device's current stream. On error the workspace is re-armed
    so that later calls start clean.
    """
    wss = [workspace_for(device)] if device is not None else list(_workspaces.values())
    for ws in wss:
        v = ws.read_errors(clear=True)
        if v:
            ws.reset()
            bits = [msg for bit, msg in _L.DEVERR.items() if v & bit]
            raise RuntimeError(f"unbox_b200 device error on {ws.device}: " + "; ".join(bits))


def _int32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int32:
        if t.dtype.is_floating_point:
            raise TypeError(f"{name} must be an integer tensor")
        t = t.to(torch.int32)
    return t


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                    context_lens: torch.Tensor, scale: Optional[float] = None, *, out: Optional[torch.Tensor] = None,
                    schedule: str = "auto", split_pages: int = 0,
                    workspace: Optional[DecodeWorkspace] = None, k_new: Optional[torch.Tensor] = None,
                    v_new: Optional[torch.Tensor] = None, overlap_previous: bool = False) -> torch.Tensor:
    """Paged GQA decode attention: out[b, h] = softmax(scale * q[b, h] K^T) V over
    the first context_lens[b] positions of sequence b (see module docstring).

    With ``k_new``/``v_new`` ((B, KVH, D) rows of the token being decoded) the
    rows are first appended at position context_lens[b] - 1, in the same launch.
    ``overlap_previous`` (fused form only) launches with programmatic dependent
    launch: pool pages start streaming while the previous kernel on the stream
    drains. Only pass it when that kernel writes neither the pool, the block
    table nor context_lens (the previous layer's attention or this layer's QKV
    projection in a decode step).
    """
    dev = _require_cuda(q, k_cache, v_cache, block_table, context_lens)
    if (k_new is None) != (v_new is None):
        raise ValueError("pass both k_new and v_new, or neither")
    if q.dim() != 3 or k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError(f"expected q (B, H, D) and caches (NB, bs, KVH, D); got {tuple(q.shape)}, "
                         f"{tuple(k_cache.shape)}, {tuple(v_cache.shape)}")
    if q.dtype not in _DTYPES or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise TypeError(f"q, k_cache, v_cache must share one of {list(_DTYPES)}; got {q.dtype}, "
                        f"{k_cache.dtype}, {v_cache.dtype}")
    if k_cache.stride() != v_cache.stride():
        raise ValueError("k_cache and v_cache must have the same strides")
    B, H, D = q.shape
    NB, bs, KVH, D2 = k_cache.shape
    if D2 != D:
        raise ValueError(f"head_dim mismatch: q {D} vs cache {D2}")
    if q.stride(-1) != 1 or k_cache.stride(-1) != 1:
        raise ValueError("the head_dim dimension must be contiguous")
    block_table = _int32(block_table, "block_table")
    context_lens = _int32(context_lens, "context_lens")
    if block_table.dim() != 2 or block_table.shape[0] != B or block_table.stride(-1) != 1:
        raise ValueError(f"block_table must be (B, max_blocks) with contiguous rows; got {tuple(block_table.shape)}")
    if context_lens.shape != (B,) or not context_lens.is_contiguous():
        raise ValueError(f"context_lens must be a contiguous ({B},) tensor")
    if out is None:
        out = torch.empty((B, H, D), dtype=q.dtype, device=dev)
    elif out.shape != (B, H, D) or out.dtype != q.dtype or out.stride(-1) != 1:
        raise ValueError("out must be (B, H, D) in q's dtype with a contiguous last dimension")
    if B == 0:
        return out
    if scale is None:
        scale = D ** -0.5
    max_blocks = block_table.shape[1]
    ws = workspace or workspace_for(dev)
    buf = ws.ensure(B, H, D, max_blocks, split_pages)
    lib = _L.load()
    tail = (block_table.data_ptr(), block_table.stride(0), context_lens.data_ptr(), out.data_ptr(), out.stride(0),
            out.stride(1), B, H, KVH, D, bs, NB, max_blocks, float(scale), _DTYPES[q.dtype], _SCHEDULES[schedule],
            int(split_pages), buf.data_ptr(), buf.numel(), _stream(dev))
    if k_new is None:
        if overlap_previous:
            raise ValueError("overlap_previous applies to the fused append + attention call")
        st = lib.ubx_paged_decode_attention(
            q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(),
            k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), *tail)
        _L.check(st, "paged_decode_attention")
    else:
        _require_cuda(q, k_new, v_new)
        if k_new.shape != (B, KVH, D) or v_new.shape != k_new.shape:
            raise ValueError(f"k_new / v_new must be ({B}, {KVH}, {D})")
        if k_new.dtype != q.dtype or v_new.dtype != q.dtype:
            raise TypeError("k_new / v_new must have the cache dtype")
        if k_new.stride() != v_new.stride() or k_new.stride(-1) != 1:
            raise ValueError("k_new and v_new need equal strides and a contiguous last dimension")
        st = lib.ubx_paged_decode_append_attention(
            k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), k_new.stride(1),
            q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(),
            k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), *tail[:-3],
            _L.FLAG_OVERLAP_PREVIOUS if overlap_previous else 0, *tail[-3:])
        _L.check(st, "paged_decode_append_attention")
    return out


def paged_decode_append_attention(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor,
                                  v_cache: torch.Tensor, block_table: torch.Tensor, context_lens: torch.Tensor,
                                  scale: Optional[float] = None, *, out: Optional[torch.Tensor] = None,
                                  schedule: str = "auto", overlap_previous: bool = False) -> torch.Tensor:
    """One decode layer's KV append and attention in one launch: the engine's
    append loop (engine.py:213-215) and attention call (:221-224)."""
    return paged_attention(q, k_cache, v_cache, block_table, context_lens, scale, out=out, schedule=schedule,
                           k_new=k_new, v_new=v_new, overlap_previous=overlap_previous)


def paged_attention_split(q, k_cache, v_cache, block_table, context_lens, scale=None, split_pages: int = 32,
                          out=None):
    """Split-KV (flash-decoding) schedule: fixed chunks of ``split_pages`` pages per
    sequence, merged by the log-sum-exp combine kernel."""
    return paged_attention(q, k_cache, v_cache, block_table, context_lens, scale, out=out, schedule="split",
                           split_pages=split_pages)


def paged_decode_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, block_tables: torch.Tensor,
                           seq_lens: torch.Tensor, block_size: int) -> torch.Tensor:
    """Drop-in for ``paged_decode_attention`` of the reference
    (paged_decode_attention.py:106-150): same positional arguments as the engine's
    call (engine.py:221-224); the softmax scale is head_dim ** -0.5 (:134)."""
    if k_pool.dim() != 4 or k_pool.shape[1] != block_size:
        raise ValueError(f"block_size {block_size} does not match k_pool {tuple(k_pool.shape)}")
    return paged_attention(q, k_pool, v_pool, block_tables, seq_lens, q.shape[-1] ** -0.5)


def kv_append(k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
              slot_mapping: torch.Tensor) -> None:
    """k_cache[slot // bs, slot % bs] = k_new[t] (and V) for every t with slot >= 0."""
    dev = _require_cuda(k_new, v_new, k_cache, v_cache, slot_mapping)
    if k_new.dim() != 3 or v_new.shape != k_new.shape or k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("expected k_new/v_new (T, KVH, D) and caches (NB, bs, KVH, D)")
    if k_new.dtype != k_cache.dtype or v_new.dtype != k_cache.dtype or v_cache.dtype != k_cache.dtype:
        raise TypeError("new rows and caches must share one dtype")
    if k_cache.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {k_cache.dtype}")
    if k_new.stride() != v_new.stride() or k_cache.stride() != v_cache.stride():
        raise ValueError("K and V tensors must have matching strides")
    T, KVH, D = k_new.shape
    NB, bs, KVH2, D2 = k_cache.shape
    if (KVH2, D2) != (KVH, D):
        raise ValueError(f"row shape {(KVH, D)} does not match cache {(KVH2, D2)}")
    if k_new.stride(-1) != 1 or k_cache.stride(-1) != 1:
        raise ValueError("the head_dim dimension must be contiguous")
    if slot_mapping.dtype != torch.int64:
        if slot_mapping.dtype.is_floating_point:
            raise TypeError("slot_mapping must be an integer tensor")
        slot_mapping = slot_mapping.to(torch.int64)
    if slot_mapping.shape != (T,) or not slot_mapping.is_contiguous():
        raise ValueError(f"slot_mapping must be a contiguous ({T},) tensor")
    ws = workspace_for(dev)
    lib = _L.load()
    st = lib.ubx_kv_append(k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), k_new.stride(1),
                           k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1),
                           k_cache.stride(2), slot_mapping.data_ptr(), T, KVH, D, bs, NB, _DTYPES[k_cache.dtype],
                           ws.error_word_ptr(), _stream(dev))
    _L.check(st, "kv_append")


def slot_mapping(block_table: torch.Tensor, positions: torch.Tensor, block_size: int,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """slot[b] = block_table[b, pos // bs] * bs + pos % bs; -1 for pos < 0 or a -1 page."""
    dev = _require_cuda(block_table, positions)
    block_table = _int32(block_table, "block_table")
    positions = _int32(positions, "positions").contiguous()
    B = positions.shape[0]
    if block_table.dim() != 2 or block_table.shape[0] != B or block_table.stride(-1) != 1:
        raise ValueError("block_table must be (B, max_blocks) with contiguous rows")
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=dev)
    lib = _L.load()
    _L.check(lib.ubx_slot_mapping(block_table.data_ptr(), block_table.stride(0), positions.data_ptr(),
                                  out.data_ptr(), B, block_table.shape[1], block_size, _stream(dev)), "slot_mapping")
    return out
