"""CPU oracle bindings. TEST INFRASTRUCTURE ONLY.

Loads ``libpaged_oracle.so`` (built from ``paged_attention_oracle.c`` by
``oracle/build.sh``) with ctypes and wraps its three entry points for numpy
arrays / CPU torch tensors. Only tests, the smoke check and the CPU-baseline leg
of bench.py import this module; the shipped library never does.

Each wrapper names the reference function it restates:
  paged_decode_attention  -> unbox_platform/infer/kernels/paged_decode_attention.py:157-191
  kv_append               -> unbox_platform/infer/kvcache.py:253-262 and :330-340
  slot_mapping            -> unbox_platform/infer/kvcache.py:338-339
  rms_norm / rotary / qk_norm_rope -> unbox_platform/model/model.py:19-48 as the
                             engine applies them (engine.py:201-210, :121-123);
                             numpy, elementwise, no C library needed
  gather_pages / scatter_pages / payload_checksum -> KVPool.serialize_blocks /
                             deserialize_blocks (kvcache.py:268-277), numpy
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpaged_oracle.so")

F32, BF16, F16 = 0, 1, 2
STATUS = {0: "ok", 1: "empty context", 2: "bad page id", 3: "bad argument", 4: "block table too short"}

_lib = None


def build(force: bool = False) -> str:
    """Compile the C oracle in place (gcc + OpenMP)."""
    if force or not os.path.exists(LIB_PATH) or (
        os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "paged_attention_oracle.c"))
    ):
        subprocess.check_call(["bash", os.path.join(_HERE, "build.sh")])
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        i64, i32, vp, dbl = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_double
        L.oracle_paged_decode_attention.argtypes = [
            vp, i64, i64, vp, vp, i64, i64, i64, vp, i64, vp, vp,
            i32, i32, i32, i32, i32, i64, i32, dbl, i32, i32]
        L.oracle_paged_decode_attention.restype = i32
        L.oracle_kv_append.argtypes = [vp, vp, i64, i64, vp, vp, i64, i64, i64, vp, i64, i32, i32, i32, i64, i32]
        L.oracle_kv_append.restype = i32
        L.oracle_slot_mapping.argtypes = [vp, i64, vp, vp, i32, i32, i32]
        L.oracle_slot_mapping.restype = i32
        L.oracle_num_threads.argtypes = []
        L.oracle_num_threads.restype = i32
        L.oracle_set_num_threads.argtypes = [i32]
        L.oracle_set_num_threads.restype = i32
        _lib = L
    return _lib


def num_threads() -> int:
    return lib().oracle_num_threads()


def use_all_cores() -> int:
    """Run the oracle's parallel regions on every core this process may use
    (whatever OMP_NUM_THREADS says); returns that thread count."""
    import os
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    return lib().oracle_set_num_threads(n)


def _np(x):
    """numpy view of a CPU torch tensor or numpy array; bf16 is viewed as uint16."""
    try:
        import torch
        if isinstance(x, torch.Tensor):
            assert x.device.type == "cpu", "oracle runs on host memory"
            if x.dtype == torch.bfloat16:
                return x.view(torch.int16).numpy().view(np.uint16)
            return x.numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x)


def _dtype_code(x) -> int:
    try:
        import torch
        if isinstance(x, torch.Tensor):
            return {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}[x.dtype]
    except ImportError:  # pragma: no cover
        pass
    a = np.asarray(x)
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.float16:
        return F16
    raise TypeError("numpy inputs must be float32 or float16 (pass bf16 as a torch tensor)")


def _strides(a: np.ndarray):
    es = a.itemsize
    return [s // es for s in a.strides]


def paged_decode_attention(q, k_cache, v_cache, block_table, context_lens, scale=None,
                           nthreads: int = 0):
    """Oracle output (B, H, D) float64 and the status code.

    Restates paged_decode_attention_ref (paged_decode_attention.py:157-191); the
    default scale is head_dim ** -0.5 as at :169.
    """
    dt = _dtype_code(q)
    qn, kn, vn = _np(q), _np(k_cache), _np(v_cache)
    bt = np.ascontiguousarray(_np(block_table), dtype=np.int32)
    cl = np.ascontiguousarray(_np(context_lens), dtype=np.int32)
    B, H, D = qn.shape
    NB, bs, KVH, D2 = kn.shape
    assert D2 == D and vn.shape == kn.shape and _strides(kn) == _strides(vn)
    assert qn.strides[-1] == qn.itemsize and kn.strides[-1] == kn.itemsize
    if scale is None:
        scale = D ** -0.5
    out = np.zeros((B, H, D), dtype=np.float64)
    qs, ks = _strides(qn), _strides(kn)
    st = lib().oracle_paged_decode_attention(
        qn.ctypes.data, qs[0], qs[1], kn.ctypes.data, vn.ctypes.data, ks[0], ks[1], ks[2],
        bt.ctypes.data, bt.shape[1] if bt.ndim == 2 else 0, cl.ctypes.data, out.ctypes.data,
        B, H, KVH, D, bs, NB, bt.shape[1] if bt.ndim == 2 else 0, float(scale), dt, nthreads)
    return out, st


def kv_append(k_new, v_new, k_cache, v_cache, slot_mapping):
    """In-place byte copy of new K/V rows into their slots; returns the status.

    Restates KVPool.write_kv / PagedKVCache.write_kv (kvcache.py:253-262, 330-340).
    """
    dt = _dtype_code(k_new)
    kn, vn = _np(k_new), _np(v_new)
    kc, vc = _np(k_cache), _np(v_cache)
    sm = np.ascontiguousarray(_np(slot_mapping), dtype=np.int64)
    T, KVH, D = kn.shape
    NB, bs, KVH2, D2 = kc.shape
    assert (KVH2, D2) == (KVH, D) and _strides(kn) == _strides(vn) and _strides(kc) == _strides(vc)
    ns, cs = _strides(kn), _strides(kc)
    return lib().oracle_kv_append(
        kn.ctypes.data, vn.ctypes.data, ns[0], ns[1], kc.ctypes.data, vc.ctypes.data,
        cs[0], cs[1], cs[2], sm.ctypes.data, T, KVH, D, bs, NB, dt)


def slot_mapping(block_table, positions, block_size: int):
    """slot[b] = block_table[b, pos // bs] * bs + pos % bs (kvcache.py:338-339)."""
    bt = np.ascontiguousarray(_np(block_table), dtype=np.int32)
    pos = np.ascontiguousarray(_np(positions), dtype=np.int32)
    out = np.empty(pos.shape[0], dtype=np.int64)
    st = lib().oracle_slot_mapping(bt.ctypes.data, bt.shape[1], pos.ctypes.data, out.ctypes.data,
                                   pos.shape[0], bt.shape[1], block_size)
    return out, st


# ---------------------------------------------------------------------------
# pre-attention (numpy): RMSNorm + rotary embedding with the dtype's rounding
# ---------------------------------------------------------------------------

def _as_f32(x):
    """float32 copy of a CPU torch tensor / numpy array and its dtype code."""
    code = _dtype_code(x)
    a = _np(x)
    if code == BF16:
        a = (np.asarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
    return np.array(a, dtype=np.float32), code


def round_to(a: np.ndarray, code: int) -> np.ndarray:
    """Round float32 values to the dtype (nearest-even) and back to float32: what
    a torch op on a 16-bit tensor does with its fp32 result."""
    a = np.asarray(a, dtype=np.float32)
    if code == F32:
        return a
    if code == F16:
        return a.astype(np.float16).astype(np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float, code: int) -> np.ndarray:
    """RMSNorm.forward (model.py:25-27) over the last axis:
    x * rsqrt(mean(x^2) + eps) * w, rounding after every tensor op (the mean as
    the fp32 sum times 1/D, rounded once)."""
    x = np.asarray(x, dtype=np.float32)
    sq = round_to(x * x, code)
    mean = round_to(sq.sum(axis=-1, keepdims=True, dtype=np.float32) * np.float32(1.0 / x.shape[-1]), code)
    r = round_to(np.float32(1.0) / np.sqrt(round_to(mean + np.float32(eps), code)), code)
    return round_to(round_to(x * r, code) * np.asarray(w, dtype=np.float32), code)


def rotary(y: np.ndarray, cos_sin: np.ndarray, code: int) -> np.ndarray:
    """apply_rotary_emb's rotate (model.py:41-46): pairs (2j, 2j+1) of the last
    axis as complex numbers times (cos + i sin), in fp32, rounded to the dtype.
    ``cos_sin`` broadcasts against y[..., ::2] with a trailing (cos, sin) axis."""
    a, b = y[..., 0::2], y[..., 1::2]
    c, s = cos_sin[..., 0], cos_sin[..., 1]
    out = np.empty_like(y)
    out[..., 0::2] = a * c - b * s
    out[..., 1::2] = a * s + b * c
    return round_to(out, code)


def qk_norm_rope(q, k, q_weight, k_weight, rope, positions, eps: float = 1e-6):
    """q (T, H, D), k (T, KVH, D): RMSNorm with q_weight / k_weight, then the rotary
    embedding at positions[t] (rows of ``rope``, (P, D/2, 2) fp32). A position
    outside [0, P) leaves its rows unrotated and is reported.
    Returns (q_out, k_out) float32 holding dtype values, and the bad-position mask."""
    qf, code = _as_f32(q)
    kf, _ = _as_f32(k)
    qw, _ = _as_f32(q_weight)
    kw, _ = _as_f32(k_weight)
    tab = np.asarray(_np(rope), dtype=np.float32)
    pos = np.asarray(_np(positions)).astype(np.int64)
    bad = (pos < 0) | (pos >= tab.shape[0])
    cs = tab[np.where(bad, 0, pos)].copy()  # (T, D/2, 2)
    cs[bad] = (1.0, 0.0)
    cs = cs[:, None, :, :]                   # broadcast over heads
    q_out = rotary(rms_norm(qf, qw, eps, code), cs, code)
    k_out = rotary(rms_norm(kf, kw, eps, code), cs, code)
    return q_out, k_out, bad


# ---------------------------------------------------------------------------
# KV page hand-off (numpy)
# ---------------------------------------------------------------------------

def _pool_np(pool):
    """(L, 2, NB, bs, KVH, D) pool as a numpy array of raw elements (bf16 as uint16)."""
    return _np(pool)


def gather_pages(pool, pages) -> bytes:
    """The payload of KVPool.serialize_blocks (kvcache.py:268-271):
    data[:, :, pages] in C order, as bytes."""
    a = _pool_np(pool)
    return np.ascontiguousarray(a[:, :, np.asarray(pages, dtype=np.int64)]).tobytes()


def scatter_pages(payload: bytes, pool, pages) -> None:
    """KVPool.deserialize_blocks (kvcache.py:273-277) with the payload read in the
    pool's own dtype: pool[:, :, pages] = payload (in place)."""
    a = _pool_np(pool)
    L, two, NB, bs, KVH, D = a.shape
    idx = np.asarray(pages, dtype=np.int64)
    a[:, :, idx] = np.frombuffer(payload, dtype=a.dtype).reshape(L, 2, len(idx), bs, KVH, D)


def payload_checksum(payload: bytes) -> int:
    """Sum over the payload's 32-bit little-endian words p[i] of p[i] * (2i + 1), mod 2^64."""
    w = np.frombuffer(payload, dtype="<u4").astype(np.uint64)
    i = np.arange(w.shape[0], dtype=np.uint64)
    with np.errstate(over="ignore"):
        return int(np.sum(w * (2 * i + 1), dtype=np.uint64))
