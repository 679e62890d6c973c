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


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """Handle of torch's current CUDA stream on ``device`` (what every op launches on)."""
    if _raw_stream is not None and device.index is not None:
        return _raw_stream(device.index)  # the same handle, without building a Stream object per call
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts):
    idx = ts[0].get_device()  # -1 for host memory
    for t in ts:
        if not t.is_cuda:
            raise ValueError("unbox_b200 ops run on CUDA tensors only (no CPU fallback)")
        if t.get_device() != idx:
            raise ValueError(f"tensors on different devices: {ts[0].device} vs {t.device}")
    return ts[0].device


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
        self._sized: set = set()  # call sizes already known to fit the current buffer

    @property
    def nbytes(self) -> int:
        return 0 if self.buf is None else self.buf.numel()

    @property
    def num_sms(self) -> int:
        if not hasattr(self, "_num_sms"):
            self._num_sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        return self._num_sms

    def ensure(self, batch: int, num_heads: int, head_dim: int, max_blocks: int, split_pages: int = 0,
               num_kv_heads: int = 0, dtype: Optional[torch.dtype] = None):
        """Grow to what a call with these sizes needs."""
        key = (batch, num_heads, head_dim, max_blocks, split_pages, num_kv_heads, dtype)
        if key in self._sized:  # the decode loop asks the same sizes every layer: answer from the cache
            return self.buf
        lib = _L.load()
        need = ctypes.c_size_t(0)
        with torch.cuda.device(self.device):
            _L.check(lib.ubx_paged_decode_workspace_size(
                batch, num_heads, num_kv_heads or num_heads, head_dim, max_blocks, split_pages,
                _DTYPES.get(dtype, _L.DTYPE_F32), ctypes.byref(need)), "workspace size")
        n = max(int(need.value), 1 << 20)
        if self.buf is None or self.buf.numel() < n:
            self.buf = torch.zeros(n, dtype=torch.uint8, device=self.device)
            _L.check(lib.ubx_workspace_init(self.buf.data_ptr(), self.buf.numel(), _stream(self.device)),
                     "workspace init")
            self._sized.clear()
        self._sized.add(key)
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
    q_st, c_st = q.stride(), k_cache.stride()
    if c_st != v_cache.stride():
        raise ValueError("k_cache and v_cache must have the same strides")
    B, H, D = q.shape
    NB, bs, KVH, D2 = k_cache.shape
    if D2 != D:
        raise ValueError(f"head_dim mismatch: q {D} vs cache {D2}")
    if q_st[2] != 1 or c_st[3] != 1:
        raise ValueError("the head_dim dimension must be contiguous")
    block_table = _int32(block_table, "block_table")
    context_lens = _int32(context_lens, "context_lens")
    bt_st = block_table.stride()
    if block_table.dim() != 2 or block_table.shape[0] != B or bt_st[1] != 1:
        raise ValueError(f"block_table must be (B, max_blocks) with contiguous rows; got {tuple(block_table.shape)}")
    if context_lens.shape != (B,) or not context_lens.is_contiguous():
        raise ValueError(f"context_lens must be a contiguous ({B},) tensor")
    if out is None:
        out = torch.empty((B, H, D), dtype=q.dtype, device=dev)
        o_st = out.stride()
    else:
        o_st = out.stride()
        if out.shape != (B, H, D) or out.dtype != q.dtype or o_st[2] != 1:
            raise ValueError("out must be (B, H, D) in q's dtype with a contiguous last dimension")
    if B == 0:
        return out
    if scale is None:
        scale = D ** -0.5
    max_blocks = block_table.shape[1]
    ws = workspace or workspace_for(dev)
    buf = ws.ensure(B, H, D, max_blocks, split_pages, KVH, q.dtype)
    lib = _L.load()
    tail = (block_table.data_ptr(), bt_st[0], context_lens.data_ptr(), out.data_ptr(), o_st[0], o_st[1],
            B, H, KVH, D, bs, NB, max_blocks, float(scale), _DTYPES[q.dtype], _SCHEDULES[schedule],
            int(split_pages), buf.data_ptr(), buf.numel(), _stream(dev))
    if k_new is None:
        if overlap_previous:
            raise ValueError("overlap_previous applies to the fused append + attention call")
        st = lib.ubx_paged_decode_attention(
            q.data_ptr(), q_st[0], q_st[1], k_cache.data_ptr(), v_cache.data_ptr(), c_st[0], c_st[1], c_st[2], *tail)
        _L.check(st, "paged_decode_attention")
    else:
        _require_cuda(q, k_new, v_new)
        if k_new.shape != (B, KVH, D) or v_new.shape != k_new.shape:
            raise ValueError(f"k_new / v_new must be ({B}, {KVH}, {D})")
        if k_new.dtype != q.dtype or v_new.dtype != q.dtype:
            raise TypeError("k_new / v_new must have the cache dtype")
        n_st = k_new.stride()
        if n_st != v_new.stride() or n_st[2] != 1:
            raise ValueError("k_new and v_new need equal strides and a contiguous last dimension")
        st = lib.ubx_paged_decode_append_attention(
            k_new.data_ptr(), v_new.data_ptr(), n_st[0], n_st[1],
            q.data_ptr(), q_st[0], q_st[1], k_cache.data_ptr(), v_cache.data_ptr(), c_st[0], c_st[1], c_st[2],
            *tail[:-3], _L.FLAG_OVERLAP_PREVIOUS if overlap_previous else 0, *tail[-3:])
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


# ---------------------------------------------------------------------------
# pre-attention: q/k RMSNorm + rotary embedding (+ KV append)
# ---------------------------------------------------------------------------

def rope_table(head_dim: int, num_positions: int, theta: float = 500000.0, device=None) -> torch.Tensor:
    """(num_positions, head_dim // 2, 2) fp32 (cos, sin) table: torch.view_as_real of
    the model's complex ``freqs_cis`` (precompute_freqs_cis, model.py:30-34; the
    engine slices it at the token positions, engine.py:108 / :206). Built on the
    CPU, like the model's buffer, then moved to ``device``."""
    freqs = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    ang = torch.outer(torch.arange(num_positions), freqs)
    tab = torch.view_as_real(torch.polar(torch.ones_like(ang), ang)).contiguous()
    return tab if device is None else tab.to(device)


def _rope_args(rope: torch.Tensor, head_dim: int):
    if rope.dtype == torch.complex64:
        rope = torch.view_as_real(rope)
    if rope.dtype != torch.float32 or rope.dim() != 3 or rope.shape[1:] != (head_dim // 2, 2):
        raise ValueError(f"rope must be (P, {head_dim // 2}, 2) float32 (cos, sin) or (P, {head_dim // 2}) complex64")
    if rope.stride(2) != 1 or rope.stride(1) != 2:
        raise ValueError("rope rows must be contiguous")
    return rope, rope.stride(0), rope.shape[0]


def _norm_weight(w: torch.Tensor, dtype, head_dim: int, name: str) -> torch.Tensor:
    if w.shape != (head_dim,) or w.dtype != dtype or not w.is_contiguous():
        raise ValueError(f"{name} must be a contiguous ({head_dim},) tensor in {dtype}")
    return w


def qk_norm_rope(q: torch.Tensor, k: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                 rope: torch.Tensor, positions: torch.Tensor, eps: float = 1e-6, *,
                 v: Optional[torch.Tensor] = None, k_cache: Optional[torch.Tensor] = None,
                 v_cache: Optional[torch.Tensor] = None, slot_mapping: Optional[torch.Tensor] = None,
                 q_out: Optional[torch.Tensor] = None, k_out: Optional[torch.Tensor] = None,
                 return_k: bool = True):
    """RMSNorm (model.py:25-27) and rotary embedding (model.py:36-48) of the q and k
    head rows of T tokens at ``positions``, as the engine's q_norm / k_norm /
    apply_rotary_emb steps (engine.py:201-210 decode, :121-123 prefill), in one
    launch. With ``k_cache``/``v_cache``/``slot_mapping`` (and ``v``) the rotated k
    row and the raw v row of every token are also stored at its slot (the write_kv
    loop, engine.py:213-215 / :126-128).

    q: (T, H, D); k, v: (T, KVH, D); weights (D,) in the model dtype; rope as
    ``rope_table``. Returns (q_out, k_out) -- k_out is None with ``return_k=False``.
    """
    dev = _require_cuda(q, k, q_weight, k_weight, rope, positions)
    if q.dim() != 3 or k.dim() != 3 or q.shape[0] != k.shape[0] or q.shape[2] != k.shape[2]:
        raise ValueError(f"expected q (T, H, D) and k (T, KVH, D); got {tuple(q.shape)}, {tuple(k.shape)}")
    if q.dtype not in _DTYPES or k.dtype != q.dtype:
        raise TypeError(f"q and k must share one of {list(_DTYPES)}")
    T, H, D = q.shape
    KVH = k.shape[1]
    if q.stride(-1) != 1 or k.stride(-1) != 1:
        raise ValueError("the head_dim dimension must be contiguous")
    q_weight = _norm_weight(q_weight, q.dtype, D, "q_weight")
    k_weight = _norm_weight(k_weight, q.dtype, D, "k_weight")
    rope, rope_sp, rope_n = _rope_args(rope, D)
    positions = _int32(positions, "positions").contiguous()
    if positions.shape != (T,):
        raise ValueError(f"positions must be ({T},)")
    if q_out is None:
        q_out = torch.empty((T, H, D), dtype=q.dtype, device=dev)
    if return_k and k_out is None:
        k_out = torch.empty((T, KVH, D), dtype=q.dtype, device=dev)
    for name, t, shp in (("q_out", q_out, (T, H, D)), ("k_out", k_out, (T, KVH, D))):
        if t is not None and (t.shape != shp or t.dtype != q.dtype or t.stride(-1) != 1):
            raise ValueError(f"{name} must be {shp} in {q.dtype} with a contiguous last dimension")
    append = k_cache is not None
    cache_args = (None, None, 0, 0, 0, None, 0, 0)
    if append:
        if v is None or v_cache is None or slot_mapping is None:
            raise ValueError("the append needs v, k_cache, v_cache and slot_mapping")
        _require_cuda(q, v, k_cache, v_cache, slot_mapping)
        if v.shape != k.shape or v.dtype != q.dtype or v.stride(-1) != 1:
            raise ValueError("v must match k")
        if k_cache.dim() != 4 or v_cache.shape != k_cache.shape or k_cache.shape[2:] != (KVH, D):
            raise ValueError(f"caches must be (NB, bs, {KVH}, {D})")
        if k_cache.dtype != q.dtype or v_cache.dtype != q.dtype or k_cache.stride() != v_cache.stride():
            raise ValueError("caches must share q's dtype and have equal strides")
        if slot_mapping.dtype != torch.int64:
            slot_mapping = slot_mapping.to(torch.int64)
        slot_mapping = slot_mapping.contiguous()
        if slot_mapping.shape != (T,):
            raise ValueError(f"slot_mapping must be ({T},)")
        NB, bs = k_cache.shape[0], k_cache.shape[1]
        cache_args = (k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1),
                      k_cache.stride(2), slot_mapping.data_ptr(), NB, bs)
    if T == 0:
        return q_out, k_out
    ws = workspace_for(dev)
    lib = _L.load()
    st = lib.ubx_qk_norm_rope_append(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1),
        v.data_ptr() if append else None, v.stride(0) if append else 0, v.stride(1) if append else 0,
        q_weight.data_ptr(), k_weight.data_ptr(), float(eps), rope.data_ptr(), rope_sp, rope_n,
        positions.data_ptr(), q_out.data_ptr(), q_out.stride(0), q_out.stride(1),
        k_out.data_ptr() if k_out is not None else None, k_out.stride(0) if k_out is not None else 0,
        k_out.stride(1) if k_out is not None else 0, *cache_args, T, H, KVH, D, _DTYPES[q.dtype],
        ws.error_word_ptr(), _stream(dev))
    _L.check(st, "qk_norm_rope_append")
    return q_out, k_out


def paged_decode_prep_attention(q_raw: torch.Tensor, k_raw: torch.Tensor, v_new: torch.Tensor,
                                q_weight: torch.Tensor, k_weight: torch.Tensor, rope: torch.Tensor,
                                k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                                context_lens: torch.Tensor, eps: float = 1e-6, scale: Optional[float] = None, *,
                                out: Optional[torch.Tensor] = None, schedule: str = "auto",
                                overlap_previous: bool = False) -> torch.Tensor:
    """The attention block of one decode layer between the QKV projection and o_proj
    (engine.py:201-224): q/k RMSNorm, rotary embedding at position
    context_lens[b] - 1, the KV append and paged attention, in one launch for
    bf16/f16. fp32 runs ``qk_norm_rope`` (with the append) and then
    ``paged_attention``: two launches.

    q_raw: (B, H, D) q projection; k_raw, v_new: (B, KVH, D) k and v projections.
    """
    dev = _require_cuda(q_raw, k_raw, v_new, q_weight, k_weight, rope, k_cache, v_cache, block_table, context_lens)
    if q_raw.dim() != 3:
        raise ValueError("q_raw must be (B, H, D)")
    B, H, D = q_raw.shape
    if q_raw.dtype == torch.float32:
        ctx = _int32(context_lens, "context_lens")
        positions = ctx - 1
        slots = slot_mapping(block_table, positions, k_cache.shape[1])
        q_rot, _ = qk_norm_rope(q_raw, k_raw, q_weight, k_weight, rope, positions, eps, v=v_new, k_cache=k_cache,
                                v_cache=v_cache, slot_mapping=slots, return_k=False)
        return paged_attention(q_rot, k_cache, v_cache, block_table, ctx, scale, out=out, schedule=schedule)
    if q_raw.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {q_raw.dtype}")
    if k_raw.shape != v_new.shape or k_raw.dim() != 3 or k_raw.shape[0] != B or k_raw.shape[2] != D:
        raise ValueError(f"k_raw / v_new must be (B, KVH, {D})")
    if k_raw.dtype != q_raw.dtype or v_new.dtype != q_raw.dtype:
        raise TypeError("k_raw / v_new must have q_raw's dtype")
    if k_raw.stride() != v_new.stride() or k_raw.stride(-1) != 1 or q_raw.stride(-1) != 1:
        raise ValueError("k_raw and v_new need equal strides; every last dimension must be contiguous")
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape or k_cache.stride() != v_cache.stride():
        raise ValueError("caches must be (NB, bs, KVH, D) with equal strides")
    if k_cache.dtype != q_raw.dtype or v_cache.dtype != q_raw.dtype:
        raise TypeError("caches must have q_raw's dtype")
    NB, bs, KVH, D2 = k_cache.shape
    if D2 != D or k_raw.shape[1] != KVH:
        raise ValueError("head shape mismatch between projections and caches")
    q_weight = _norm_weight(q_weight, q_raw.dtype, D, "q_weight")
    k_weight = _norm_weight(k_weight, q_raw.dtype, D, "k_weight")
    rope, rope_sp, rope_n = _rope_args(rope, D)
    block_table = _int32(block_table, "block_table")
    context_lens = _int32(context_lens, "context_lens")
    if block_table.dim() != 2 or block_table.shape[0] != B or block_table.stride(-1) != 1:
        raise ValueError("block_table must be (B, max_blocks) with contiguous rows")
    if context_lens.shape != (B,) or not context_lens.is_contiguous():
        raise ValueError(f"context_lens must be a contiguous ({B},) tensor")
    if out is None:
        out = torch.empty((B, H, D), dtype=q_raw.dtype, device=dev)
    elif out.shape != (B, H, D) or out.dtype != q_raw.dtype or out.stride(-1) != 1:
        raise ValueError("out must be (B, H, D) in q's dtype with a contiguous last dimension")
    if B == 0:
        return out
    if scale is None:
        scale = D ** -0.5
    max_blocks = block_table.shape[1]
    buf = workspace_for(dev).ensure(B, H, D, max_blocks, 0, KVH, q_raw.dtype)
    lib = _L.load()
    st = lib.ubx_paged_decode_prep_attention(
        q_raw.data_ptr(), q_raw.stride(0), q_raw.stride(1), k_raw.data_ptr(), v_new.data_ptr(), k_raw.stride(0),
        k_raw.stride(1), q_weight.data_ptr(), k_weight.data_ptr(), float(eps), rope.data_ptr(), rope_sp, rope_n,
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
        block_table.data_ptr(), block_table.stride(0), context_lens.data_ptr(), out.data_ptr(), out.stride(0),
        out.stride(1), B, H, KVH, D, bs, NB, max_blocks, float(scale), _DTYPES[q_raw.dtype], _SCHEDULES[schedule],
        0, _L.FLAG_OVERLAP_PREVIOUS if overlap_previous else 0, buf.data_ptr(), buf.numel(), _stream(dev))
    _L.check(st, "paged_decode_prep_attention")
    return out


# ---------------------------------------------------------------------------
# prefill: the chunk's KV rows written in one launch
# ---------------------------------------------------------------------------

def prefill_slots(block_table_row: torch.Tensor, start_pos: int, num_tokens: int, block_size: int) -> torch.Tensor:
    """Slots of positions start_pos .. start_pos + num_tokens - 1 of one sequence
    (kvcache.py:338-339 for every token of a prefill chunk)."""
    dev = _require_cuda(block_table_row)
    row = _int32(block_table_row, "block_table_row").contiguous()
    if row.dim() != 1:
        raise ValueError("block_table_row must be 1-D")
    positions = torch.arange(start_pos, start_pos + num_tokens, dtype=torch.int32, device=dev)
    return slot_mapping(row.unsqueeze(0).expand(num_tokens, -1), positions, block_size)


def prefill_kv_write(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     block_table_row: torch.Tensor, start_pos: int, *, overlap_previous: bool = False) -> torch.Tensor:
    """Write the K/V rows of a prefill chunk (T tokens of one sequence starting at
    ``start_pos``) into the pool: the per-token write_kv loop of prefill_step
    (engine.py:126-128) as one launch that computes each token's slot from the
    block-table row and copies its rows. Returns the slots (T,) int64.
    ``overlap_previous``: programmatic dependent launch (the launch overlaps the
    previous kernel's drain; nothing is touched before that kernel completes)."""
    dev = _require_cuda(k, v, k_cache, v_cache, block_table_row)
    if k.dim() != 3 or v.shape != k.shape or k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("expected k/v (T, KVH, D) and caches (NB, bs, KVH, D)")
    if k.dtype != k_cache.dtype or v.dtype != k_cache.dtype or v_cache.dtype != k_cache.dtype:
        raise TypeError("chunk rows and caches must share one dtype")
    if k_cache.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {k_cache.dtype}")
    if k.stride() != v.stride() or k_cache.stride() != v_cache.stride():
        raise ValueError("K and V tensors must have matching strides")
    T, KVH, D = k.shape
    NB, bs, KVH2, D2 = k_cache.shape
    if (KVH2, D2) != (KVH, D):
        raise ValueError(f"row shape {(KVH, D)} does not match cache {(KVH2, D2)}")
    if k.stride(-1) != 1 or k_cache.stride(-1) != 1:
        raise ValueError("the head_dim dimension must be contiguous")
    row = _int32(block_table_row, "block_table_row").contiguous()
    if row.dim() != 1:
        raise ValueError("block_table_row must be 1-D")
    if start_pos < 0:
        raise ValueError("start_pos must be >= 0")
    slots = torch.empty(T, dtype=torch.int64, device=dev)
    if T == 0:
        return slots
    ws = workspace_for(dev)
    st = _L.load().ubx_prefill_kv_write(k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k_cache.data_ptr(),
                                        v_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
                                        row.data_ptr(), row.shape[0], int(start_pos), T, KVH, D, bs, NB,
                                        _DTYPES[k_cache.dtype], slots.data_ptr(), ws.error_word_ptr(),
                                        _L.FLAG_OVERLAP_PREVIOUS if overlap_previous else 0, _stream(dev))
    _L.check(st, "prefill_kv_write")
    return slots


def prefill_positions_and_slots(block_table_row: torch.Tensor, start_pos: int, num_tokens: int,
                                block_size: int = 16):
    """Positions start_pos .. and their KV slots for a prefill chunk; the same for
    every layer of the step, so computed once and passed to ``prefill_prep``."""
    row = _int32(block_table_row, "block_table_row").contiguous()
    if row.dim() != 1:
        raise ValueError("block_table_row must be 1-D")
    positions = torch.arange(start_pos, start_pos + num_tokens, dtype=torch.int32, device=row.device)
    return positions, slot_mapping(row.unsqueeze(0).expand(num_tokens, -1), positions, block_size)


def prefill_prep(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                 rope: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table_row: torch.Tensor,
                 start_pos: int, eps: float = 1e-6, positions_and_slots=None):
    """A prefill chunk's q_norm / k_norm / rotary embedding at positions
    start_pos.. and its KV write (engine.py:121-128) in one launch (plus the slot
    computation, unless ``positions_and_slots`` -- from
    ``prefill_positions_and_slots``, once per step -- is given). Returns (q_rot,
    k_rot) for the chunk's own attention."""
    T = q.shape[0]
    _require_cuda(q)
    if positions_and_slots is None:
        positions_and_slots = prefill_positions_and_slots(block_table_row, start_pos, T, k_cache.shape[1])
    positions, slots = positions_and_slots
    if positions.shape != (T,) or slots.shape != (T,):
        raise ValueError(f"positions and slots must hold the chunk's {T} tokens")
    return qk_norm_rope(q, k, q_weight, k_weight, rope, positions, eps, v=v, k_cache=k_cache, v_cache=v_cache,
                        slot_mapping=slots)
