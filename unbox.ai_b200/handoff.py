"""KV page hand-off between a prefill worker and a decode worker, on the device.

Mirrors the reference's transfer path (unbox_platform/infer/kvcache.py:268-277,
worker.py:175-183 and :217-223):

* ``serialize_blocks(pool_data, block_indices) -> bytes`` -- KVPool.serialize_blocks:
  the pages of every layer, K and V, in the reference's byte order
  ``data[:, :, block_indices]``, behind a 64-byte header that names the dtype and
  geometry and carries a checksum. The gather runs on the GPU; only the finished
  message crosses to the host.
* ``deserialize_blocks(pool_data, data, block_indices)`` -- KVPool.deserialize_blocks:
  checks the header against the pool, checks the checksum, and scatters the
  pages into ``block_indices`` of this pool (the decode worker's own pages).
  Unlike the reference it reads the payload in the pool's dtype (the reference
  decodes every payload as float32, and cannot serialise a bf16 pool at all).
* ``pack_pages`` / ``unpack_pages`` -- the same on device tensors, no host copy.
* ``transfer_pages(src_pool, src_pages, dst_pool, dst_pages)`` -- pool to pool
  in one kernel; the destination may live on another GPU (peer access): the page
  rows cross NVLink as stores, with no staging buffer, host copy or socket.
* ``ipc_export`` / ``ipc_import`` -- CUDA IPC of a pool, for worker processes
  that each own one GPU.

``pool_data`` is ``KVPool.data``: (num_layers, 2, num_blocks, block_size,
num_kv_heads, head_dim), contiguous pages. Every op runs on the pool's device,
on torch's current stream, and raises without the CUDA library (no fallback).
"""
from __future__ import annotations

import ctypes
import warnings
from typing import Optional, Sequence, Union

import torch

from . import library as _L
from .ops import _DTYPES, _require_cuda, _stream, workspace_for

HEADER_BYTES = 64


def _geometry(pool: torch.Tensor):
    if pool.dim() != 6 or pool.shape[1] != 2:
        raise ValueError(f"pool must be KVPool.data (L, 2, NB, bs, KVH, D); got {tuple(pool.shape)}")
    if pool.dtype not in _DTYPES:
        raise TypeError(f"unsupported pool dtype {pool.dtype}")
    L, _, NB, bs, KVH, D = pool.shape
    if pool.stride(5) != 1 or pool.stride(4) != D or pool.stride(3) != KVH * D:
        raise ValueError("pool pages must be contiguous (block_size, num_kv_heads, head_dim) blocks")
    return L, NB, bs, KVH, D


def _pages(pages, device) -> torch.Tensor:
    if isinstance(pages, torch.Tensor):
        t = pages.to(device=device, dtype=torch.int32)
    else:
        t = torch.tensor(list(pages), dtype=torch.int32, device=device)
    return t.contiguous()


def _copy(src, src_strides, src_pages, src_nb, dst, dst_strides, dst_pages, dst_nb, L, n, page_elems, dtype,
          checksum=None, device=None):
    lib = _L.load()
    ws = workspace_for(device)
    st = lib.ubx_kv_pages_copy(
        src.data_ptr(), *src_strides, None if src_pages is None else src_pages.data_ptr(), src_nb,
        dst.data_ptr(), *dst_strides, None if dst_pages is None else dst_pages.data_ptr(), dst_nb,
        L, n, page_elems, _DTYPES[dtype], None if checksum is None else checksum.data_ptr(),
        ws.error_word_ptr(), _stream(device))
    _L.check(st, "kv_pages_copy")


def _packed_strides(n: int, page_elems: int):
    return (2 * n * page_elems, n * page_elems, page_elems)


def pack_pages(pool: torch.Tensor, pages, out: Optional[torch.Tensor] = None,
               checksum: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gather ``pages`` of every layer (K and V) into a packed payload
    (L, 2, n, bs, KVH, D) on the pool's device. With ``checksum`` (a device int64
    tensor of one element) the payload checksum lands there too."""
    dev = _require_cuda(pool)
    L, NB, bs, KVH, D = _geometry(pool)
    idx = _pages(pages, dev)
    n = idx.numel()
    if out is None:
        out = torch.empty((L, 2, n, bs, KVH, D), dtype=pool.dtype, device=dev)
    elif out.shape != (L, 2, n, bs, KVH, D) or out.dtype != pool.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous (L, 2, n, bs, KVH, D) tensor of the pool dtype")
    pe = bs * KVH * D
    _copy(pool, (pool.stride(0), pool.stride(1), pool.stride(2)), idx, NB, out, _packed_strides(n, pe), None, 0,
          L, n, pe, pool.dtype, checksum, dev)
    return out


def unpack_pages(payload: torch.Tensor, pool: torch.Tensor, pages, checksum: Optional[torch.Tensor] = None) -> None:
    """Scatter a packed payload (L, 2, n, bs, KVH, D) into ``pages`` of ``pool``
    (in place); ``checksum`` receives the payload checksum as read."""
    dev = _require_cuda(pool, payload)
    L, NB, bs, KVH, D = _geometry(pool)
    idx = _pages(pages, dev)
    n = idx.numel()
    if payload.shape != (L, 2, n, bs, KVH, D) or payload.dtype != pool.dtype or not payload.is_contiguous():
        raise ValueError(f"payload must be a contiguous {(L, 2, n, bs, KVH, D)} tensor of the pool dtype")
    pe = bs * KVH * D
    _copy(payload, _packed_strides(n, pe), None, 0, pool, (pool.stride(0), pool.stride(1), pool.stride(2)), idx, NB,
          L, n, pe, pool.dtype, checksum, dev)


def make_header(pool: torch.Tensor, num_pages: int, checksum: int) -> bytes:
    L, NB, bs, KVH, D = _geometry(pool)
    h = _L.KVWireHeader()
    _L.check(_L.load().ubx_kv_wire_header_init(ctypes.byref(h), _DTYPES[pool.dtype], L, KVH, D, bs, num_pages,
                                                ctypes.c_uint64(checksum & (2 ** 64 - 1))), "kv wire header")
    return bytes(h)


def parse_header(data: Union[bytes, bytearray, memoryview]) -> _L.KVWireHeader:
    if len(data) < HEADER_BYTES:
        raise ValueError(f"message of {len(data)} bytes is shorter than the {HEADER_BYTES}-byte header")
    return _L.KVWireHeader.from_buffer_copy(bytes(data[:HEADER_BYTES]))


def check_header(h: _L.KVWireHeader, pool: torch.Tensor, payload_bytes: int) -> None:
    L, NB, bs, KVH, D = _geometry(pool)
    _L.check(_L.load().ubx_kv_wire_header_check(ctypes.byref(h), _DTYPES[pool.dtype], L, KVH, D, bs,
                                                 ctypes.c_uint64(payload_bytes)), "kv wire header")


def _u64(t: torch.Tensor) -> int:
    return int(t.item()) & (2 ** 64 - 1)


def serialize_blocks(pool: torch.Tensor, block_indices: Sequence[int]) -> bytearray:
    """KVPool.serialize_blocks (kvcache.py:268-271): header + the pages' bytes, as
    one bytes-like message that the device-to-host copy writes in place.
    Synchronises the stream (the message is host memory)."""
    dev = _require_cuda(pool)
    ck = torch.zeros(1, dtype=torch.int64, device=dev)
    payload = pack_pages(pool, block_indices, checksum=ck)
    nbytes = payload.numel() * payload.element_size()
    msg = bytearray(HEADER_BYTES + nbytes)
    if nbytes:
        body = torch.frombuffer(msg, dtype=torch.uint8, offset=HEADER_BYTES, count=nbytes)
        body.copy_(payload.view(-1).view(torch.uint8))
    torch.cuda.current_stream(dev).synchronize()
    msg[:HEADER_BYTES] = make_header(pool, len(block_indices), _u64(ck))
    return msg


def deserialize_blocks(pool: torch.Tensor, data: Union[bytes, bytearray, memoryview],
                       block_indices: Sequence[int], verify: bool = True) -> None:
    """KVPool.deserialize_blocks (kvcache.py:273-277) for messages made by
    ``serialize_blocks``: the header must match this pool's dtype and geometry,
    the pages land in ``block_indices`` of this pool, and with ``verify`` the
    checksum of the bytes as scattered must equal the header's (synchronises)."""
    dev = _require_cuda(pool)
    h = parse_header(data)
    body = memoryview(data)[HEADER_BYTES:]
    check_header(h, pool, len(body))
    if h.num_pages != len(block_indices):
        raise ValueError(f"message holds {h.num_pages} pages, {len(block_indices)} destinations given")
    L, NB, bs, KVH, D = _geometry(pool)
    staged = torch.empty(len(body), dtype=torch.uint8, device=dev)
    if len(body):
        with warnings.catch_warnings():  # read-only buffers (bytes) are only read here
            warnings.simplefilter("ignore", UserWarning)
            host = torch.frombuffer(data, dtype=torch.uint8, offset=HEADER_BYTES, count=len(body))
        staged.copy_(host)
    payload = staged.view(pool.dtype).view(L, 2, h.num_pages, bs, KVH, D)
    ck = torch.zeros(1, dtype=torch.int64, device=dev) if verify else None
    unpack_pages(payload, pool, block_indices, checksum=ck)
    if verify and _u64(ck) != int(h.checksum):
        raise RuntimeError(f"KV page message checksum mismatch: {_u64(ck):#x} != header {int(h.checksum):#x}")


def transfer_pages(src_pool: torch.Tensor, src_pages, dst_pool: torch.Tensor, dst_pages, on: str = "source") -> None:
    """Copy ``src_pages`` of every layer of ``src_pool`` into ``dst_pages`` of
    ``dst_pool`` with one kernel, on the source device (``on="source"``: a
    prefill worker pushing) or on the destination device (``on="destination"``:
    a decode worker pulling), on torch's current stream there. When the pools
    sit on different GPUs that kernel reaches the other pool over NVLink with
    plain loads or stores (peer access is enabled on first use); the caller
    orders later use of the pages on the other GPU after this stream (e.g. an
    event)."""
    if on not in ("source", "destination"):
        raise ValueError("on must be 'source' or 'destination'")
    _require_cuda(src_pool)
    if dst_pool.device.type != "cuda":
        raise ValueError("dst_pool must be a CUDA tensor")
    g1, g2 = _geometry(src_pool), _geometry(dst_pool)
    if g1[0] != g2[0] or g1[2:] != g2[2:] or src_pool.dtype != dst_pool.dtype:
        raise ValueError("source and destination pools differ in dtype or page geometry")
    L, NB, bs, KVH, D = g1
    run, other = (src_pool.device, dst_pool.device) if on == "source" else (dst_pool.device, src_pool.device)
    si, di = _pages(src_pages, run), _pages(dst_pages, run)
    if si.numel() != di.numel():
        raise ValueError("as many destination pages as source pages")
    with torch.cuda.device(run):
        if other != run:
            _L.check(_L.load().ubx_enable_peer_access(other.index), "enable peer access")
        _copy(src_pool, (src_pool.stride(0), src_pool.stride(1), src_pool.stride(2)), si, NB,
              dst_pool, (dst_pool.stride(0), dst_pool.stride(1), dst_pool.stride(2)), di, g2[1], L, si.numel(),
              bs * KVH * D, src_pool.dtype, None, run)


# ---------------------------------------------------------------------------
# CUDA IPC: one process per GPU
# ---------------------------------------------------------------------------

def ipc_export(t: torch.Tensor) -> bytes:
    """72-byte token for ``t``'s memory: the 64-byte CUDA IPC handle of its
    allocation and t's byte offset in it."""
    _require_cuda(t)
    handle = (ctypes.c_uint8 * 64)()
    off = ctypes.c_uint64(0)
    with torch.cuda.device(t.device):
        _L.check(_L.load().ubx_ipc_get_handle(t.data_ptr(), handle, ctypes.byref(off)), "ipc handle")
    return bytes(handle) + int(off.value).to_bytes(8, "little")


class IpcMapping:
    """A peer process's buffer mapped into this process (``ipc_import``):
    ``ptr`` is the device address of the exported tensor's first byte."""

    def __init__(self, token: bytes, device: torch.device):
        self.device = torch.device(device)
        base = ctypes.c_void_p(0)
        handle = (ctypes.c_uint8 * 64).from_buffer_copy(token[:64])
        with torch.cuda.device(self.device):
            _L.check(_L.load().ubx_ipc_open_handle(handle, ctypes.byref(base)), "ipc open")
        self._base = base.value
        self.ptr = self._base + int.from_bytes(token[64:72], "little")

    def close(self):
        if self._base:
            with torch.cuda.device(self.device):
                _L.check(_L.load().ubx_ipc_close_handle(ctypes.c_void_p(self._base)), "ipc close")
            self._base = 0


def ipc_import(token: bytes, device) -> IpcMapping:
    return IpcMapping(token, device)


def transfer_pages_to_ipc(src_pool: torch.Tensor, src_pages, dst: IpcMapping, dst_shape, dst_pages) -> None:
    """``transfer_pages`` into a pool of another process, mapped by ``ipc_import``
    (``dst_shape`` = that pool's (L, 2, NB, bs, KVH, D), contiguous)."""
    sdev = _require_cuda(src_pool)
    L, NB, bs, KVH, D = _geometry(src_pool)
    L2, two, NB2, bs2, KVH2, D2 = dst_shape
    if (L2, two, bs2, KVH2, D2) != (L, 2, bs, KVH, D):
        raise ValueError("destination pool geometry differs")
    si, di = _pages(src_pages, sdev), _pages(dst_pages, sdev)
    if si.numel() != di.numel():
        raise ValueError("as many destination pages as source pages")
    pe = bs * KVH * D
    dst_strides = (2 * NB2 * pe, NB2 * pe, pe)

    class _Ptr:  # the mapped address, in the shape _copy expects
        def __init__(self, p):
            self.p = p

        def data_ptr(self):
            return self.p

    with torch.cuda.device(sdev):
        _copy(src_pool, (src_pool.stride(0), src_pool.stride(1), src_pool.stride(2)), si, NB, _Ptr(dst.ptr),
              dst_strides, di, NB2, L, si.numel(), pe, src_pool.dtype, None, sdev)
