"""Seeded synthetic decode-step workloads.

A workload is the state one decode step of the unbox.ai engine hands to the
attention path: per-sequence context lengths (``seq_lens`` at
``unbox_platform/infer/engine.py:185`` -- they include the token being decoded),
a ``(B, max_blocks)`` int32 block table padded with -1 (``engine.py:179-184``),
the paged K/V pools in the ``KVPool`` layout ``(num_blocks, 16, KVH, D)``
(``unbox_platform/infer/kvcache.py:248-251,264-266``), the query of the new
token and its K/V row, which is appended at position ``ctx - 1`` before
attention runs (``engine.py:213-224``).

Layout (which pages a sequence owns) is generated with a portable counter-based
generator (splitmix64 -> Box-Muller, quantised to a 2^-16 grid) so the same seed
gives the same bytes on every host; that is what the committed golden fixtures
rely on. Tensor values for large workloads are drawn on the GPU with torch's
generator instead (``materialize_device``), which is fast and deterministic per
GPU type.

Shapes of the named workloads (GQA 16/8, head_dim 112, page 16 throughout):
  decode_760m   B=64, ctx ~ U[512, 2048], bf16, values N(0,1)*0.5
  correctness   B=8, ctx ~ U[64, 512], fp32, N(0,1), 512-page pool
  long_context  B=16, ctx ~ U[16384, 32768], bf16, N(0,1)
  radix_prefix  128 requests sharing 96 pages (1536 tokens) + U[64, 512] private tokens
  box_scale     1024 sequences, ctx log-normal (median 1024, sigma 0.6) clipped to [128, 4096]
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    x = (x + np.uint64(0x9E3779B97F4A7C15)) & _M64
    z = x
    z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & _M64
    z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & _M64
    return z ^ (z >> np.uint64(31))


def _stream(seed: int, stream: int, n: int) -> np.ndarray:
    """n uint64 words of the counter-based stream (seed, stream)."""
    base = _splitmix64(np.array([(seed * 0x632BE59BD9B4E019 + stream * 0x8CB92BA72F3D8DD7) & 0xFFFFFFFFFFFFFFFF],
                                dtype=np.uint64))[0]
    with np.errstate(over="ignore"):
        ctr = base + np.arange(n, dtype=np.uint64)
    return _splitmix64(ctr)


def portable_uniform(seed: int, stream: int, n: int) -> np.ndarray:
    """n doubles in [0, 1) with 53 random bits each."""
    return (_stream(seed, stream, n) >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)


def portable_randint(seed: int, stream: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive: the workloads' U[lo, hi] ranges)."""
    span = np.uint64(hi - lo + 1)
    return (lo + (_stream(seed, stream, n) % span).astype(np.int64)).astype(np.int64)


def portable_normal(seed: int, stream: int, n: int) -> np.ndarray:
    """n N(0,1) samples (Box-Muller), rounded to a 2^-16 grid so that a last-ulp
    difference between hosts' libm never changes the stored value."""
    w = _stream(seed, stream, 2 * n)
    u1 = ((w[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (2.0 ** -53)
    u2 = (w[1::2] >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * math.pi * u2)
    return np.round(z * 65536.0) / 65536.0


def portable_permutation(seed: int, stream: int, n: int) -> np.ndarray:
    keys = _stream(seed, stream, n)
    return np.argsort(keys, kind="stable").astype(np.int64)


@dataclasses.dataclass
class Layout:
    """Paging metadata of one decode step (host arrays)."""
    context_lens: np.ndarray          # (B,) int32, includes the token being decoded
    block_table: np.ndarray           # (B, max_blocks) int32, -1 padded
    num_blocks: int                   # pages in the pool
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 112
    block_size: int = 16
    unique_pages: Optional[int] = None  # pages referenced at least once (radix sharing)
    unique_pages_tokens: int = 0        # token rows in those pages that some sequence reads

    @property
    def batch(self) -> int:
        return int(self.context_lens.shape[0])

    @property
    def max_blocks(self) -> int:
        return int(self.block_table.shape[1])

    def positions(self) -> np.ndarray:
        """Position of the token being appended: ctx - 1 (engine.py:186-187, 213-215)."""
        return (self.context_lens.astype(np.int64) - 1).astype(np.int32)

    def slot_mapping(self) -> np.ndarray:
        """slot = block_table[b, pos // bs] * bs + pos % bs (kvcache.py:338-339);
        -1 (padding, nothing appended) for an empty context or a -1 page."""
        pos = self.positions().astype(np.int64)
        out = np.full(self.batch, -1, dtype=np.int64)
        ok = pos >= 0
        b = np.arange(self.batch)[ok]
        pages = self.block_table[b, pos[ok] // self.block_size].astype(np.int64)
        out[ok] = np.where(pages >= 0, pages * self.block_size + pos[ok] % self.block_size, -1)
        return out

    def kv_tokens(self) -> int:
        """Σ ctx: token rows one attention call reads per KV head."""
        return int(self.context_lens.astype(np.int64).sum())

    def unique_kv_tokens(self) -> int:
        """Token rows counted once per physical page slot (radix prefixes counted once)."""
        if self.unique_pages is None:
            return self.kv_tokens()
        return int(self.unique_pages_tokens)


def _assign_pages(ctx: np.ndarray, perm: np.ndarray, block_size: int, max_blocks: Optional[int] = None):
    pages = (ctx + block_size - 1) // block_size
    mb = int(pages.max()) if max_blocks is None else max_blocks
    bt = np.full((ctx.shape[0], max(mb, 1)), -1, dtype=np.int32)
    cur = 0
    for b in range(ctx.shape[0]):
        n = int(pages[b])
        bt[b, :n] = perm[cur:cur + n]
        cur += n
    return bt, cur


def layout_uniform(seed: int, batch: int, ctx_lo: int, ctx_hi: int, num_blocks: Optional[int] = None,
                   num_heads=16, num_kv_heads=8, head_dim=112, block_size=16) -> Layout:
    """B sequences with ctx ~ U[lo, hi]; pages are a random permutation of the
    pool handed out to sequences in order (seed-determined)."""
    ctx = portable_randint(seed, 1, batch, ctx_lo, ctx_hi).astype(np.int32)
    need = int(((ctx.astype(np.int64) + block_size - 1) // block_size).sum())
    nb = need if num_blocks is None else num_blocks
    assert nb >= need, f"pool of {nb} pages cannot hold {need}"
    perm = portable_permutation(seed, 2, nb)
    bt, _ = _assign_pages(ctx.astype(np.int64), perm, block_size)
    return Layout(ctx, bt, nb, num_heads, num_kv_heads, head_dim, block_size)


def layout_radix_prefix(seed: int, batch: int = 128, prefix_pages: int = 96, suffix_lo: int = 64,
                        suffix_hi: int = 512, block_size: int = 16) -> Layout:
    """Requests that share the same physical prefix pages (a radix-cache hit,
    kvcache.py:97-122) followed by private pages."""
    suffix = portable_randint(seed, 3, batch, suffix_lo, suffix_hi)
    ctx = (prefix_pages * block_size + suffix).astype(np.int32)
    priv_pages = (suffix + block_size - 1) // block_size
    nb = prefix_pages + int(priv_pages.sum())
    perm = portable_permutation(seed, 2, nb)
    shared = perm[:prefix_pages]
    mb = prefix_pages + int(priv_pages.max())
    bt = np.full((batch, mb), -1, dtype=np.int32)
    cur = prefix_pages
    for b in range(batch):
        bt[b, :prefix_pages] = shared
        n = int(priv_pages[b])
        bt[b, prefix_pages:prefix_pages + n] = perm[cur:cur + n]
        cur += n
    lay = Layout(ctx, bt, nb, block_size=block_size, unique_pages=nb)
    lay.unique_pages_tokens = prefix_pages * block_size + int(suffix.sum())
    return lay


def layout_lognormal(seed: int, batch: int = 1024, median: float = 1024.0, sigma: float = 0.6,
                     lo: int = 128, hi: int = 4096, block_size: int = 16) -> Layout:
    z = portable_normal(seed, 4, batch)
    ctx = np.clip(np.round(median * np.exp(sigma * z)), lo, hi).astype(np.int32)
    need = int(((ctx.astype(np.int64) + block_size - 1) // block_size).sum())
    perm = portable_permutation(seed, 2, need)
    bt, _ = _assign_pages(ctx.astype(np.int64), perm, block_size)
    return Layout(ctx, bt, need, block_size=block_size)


NAMED = {
    "correctness": dict(kind="uniform", batch=8, ctx=(64, 512), num_blocks=512, dtype="float32", scale_values=1.0),
    "decode_760m": dict(kind="uniform", batch=64, ctx=(512, 2048), num_blocks=None, dtype="bfloat16", scale_values=0.5),
    "long_context": dict(kind="uniform", batch=16, ctx=(16384, 32768), num_blocks=None, dtype="bfloat16", scale_values=1.0),
    "radix_prefix": dict(kind="radix", dtype="bfloat16", scale_values=1.0),
    "box_scale": dict(kind="lognormal", dtype="bfloat16", scale_values=1.0),
}


def named_layout(name: str, seed: int = 0) -> Layout:
    spec = NAMED[name]
    if spec["kind"] == "uniform":
        return layout_uniform(seed, spec["batch"], spec["ctx"][0], spec["ctx"][1], spec["num_blocks"])
    if spec["kind"] == "radix":
        return layout_radix_prefix(seed)
    return layout_lognormal(seed)


# ---------------------------------------------------------------------------
# tensors
# ---------------------------------------------------------------------------

def _torch_dtype(name: str):
    import torch
    return {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[name]


def materialize_host(lay: Layout, seed: int, dtype: str = "float32", value_scale: float = 1.0):
    """Host torch tensors from the portable generator (bit-identical on every host).

    Returns dict(q, k_cache, v_cache, k_new, v_new, block_table, context_lens, slot_mapping).
    """
    import torch
    B, H, KVH, D, bs, NB = lay.batch, lay.num_heads, lay.num_kv_heads, lay.head_dim, lay.block_size, lay.num_blocks
    td = _torch_dtype(dtype)

    def gen(stream, shape):
        n = int(np.prod(shape))
        a = (portable_normal(seed, stream, n) * value_scale).astype(np.float32).reshape(shape)
        return torch.from_numpy(a).to(td)

    return dict(
        q=gen(10, (B, H, D)),
        k_cache=gen(11, (NB, bs, KVH, D)),
        v_cache=gen(12, (NB, bs, KVH, D)),
        k_new=gen(13, (B, KVH, D)),
        v_new=gen(14, (B, KVH, D)),
        block_table=torch.from_numpy(lay.block_table.copy()),
        context_lens=torch.from_numpy(lay.context_lens.copy()),
        slot_mapping=torch.from_numpy(lay.slot_mapping()),
    )


def materialize_prep_host(seed: int, num_tokens: int, num_heads: int, num_kv_heads: int, head_dim: int,
                          dtype: str = "bfloat16", value_scale: float = 1.0):
    """Inputs of the pre-attention step from the portable generator: the q, k and v
    projections of ``num_tokens`` tokens and the q_norm / k_norm weights
    (1 + 0.1 N(0, 1), trained RMSNorm weights sit near 1).

    Returns dict(q_raw (T, H, D), k_raw (T, KVH, D), v_new (T, KVH, D), q_weight (D,), k_weight (D,)).
    """
    import torch
    td = _torch_dtype(dtype)

    def gen(stream, shape, scale=value_scale, offset=0.0):
        n = int(np.prod(shape))
        a = (portable_normal(seed, stream, n) * scale + offset).astype(np.float32).reshape(shape)
        return torch.from_numpy(a).to(td)

    T, H, KVH, D = num_tokens, num_heads, num_kv_heads, head_dim
    return dict(q_raw=gen(20, (T, H, D)), k_raw=gen(21, (T, KVH, D)), v_new=gen(22, (T, KVH, D)),
                q_weight=gen(23, (D,), 0.1, 1.0), k_weight=gen(24, (D,), 0.1, 1.0))


def materialize_pool_host(seed: int, num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int,
                          head_dim: int, dtype: str = "float32", stream: int = 30):
    """A whole KVPool.data tensor (L, 2, NB, bs, KVH, D) (kvcache.py:248-251) from
    the portable generator."""
    import torch
    shape = (num_layers, 2, num_blocks, block_size, num_kv_heads, head_dim)
    a = portable_normal(seed, stream, int(np.prod(shape))).astype(np.float32).reshape(shape)
    return torch.from_numpy(a).to(_torch_dtype(dtype))


def materialize_device(lay: Layout, seed: int, dtype: str, value_scale: float, num_layers: int,
                       device="cuda"):
    """Device tensors for a multi-layer decode step drawn with torch's generator.

    Returns dict with per-layer lists k_caches / v_caches / q / k_new / v_new and
    the shared block_table, context_lens, slot_mapping (one block table serves
    every layer, as in the engine).
    """
    import torch
    B, H, KVH, D, bs, NB = lay.batch, lay.num_heads, lay.num_kv_heads, lay.head_dim, lay.block_size, lay.num_blocks
    td = _torch_dtype(dtype)
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def rnd(shape):
        t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        if value_scale != 1.0:
            t.mul_(value_scale)
        return t.to(td)

    out = dict(k_caches=[], v_caches=[], q=[], k_new=[], v_new=[])
    for _ in range(num_layers):
        # one allocation per layer holding K and V, like KVPool.data[l] (kvcache.py:248-251)
        kv = torch.empty((2, NB, bs, KVH, D), device=device, dtype=td)
        for i in range(2):
            for c0 in range(0, NB, 4096):
                c1 = min(NB, c0 + 4096)
                kv[i, c0:c1].copy_(rnd((c1 - c0, bs, KVH, D)))
        out["k_caches"].append(kv[0])
        out["v_caches"].append(kv[1])
        out["q"].append(rnd((B, H, D)))
        out["k_new"].append(rnd((B, KVH, D)))
        out["v_new"].append(rnd((B, KVH, D)))
    out["block_table"] = torch.from_numpy(lay.block_table.copy()).to(device)
    out["context_lens"] = torch.from_numpy(lay.context_lens.copy()).to(device)
    out["slot_mapping"] = torch.from_numpy(lay.slot_mapping()).to(device)
    return out


def algorithmic_bytes(lay: Layout, elem_bytes: int, unique: bool = True) -> dict:
    """Bytes one layer-call must move (the roofline numerator).

    K and V rows are counted once per (sequence, KV head) because the GQA group
    shares them: Σctx * KVH * D * 2 (K and V) * elem bytes, plus q and out, the
    block-table rows the sequences use and context_lens. With ``unique`` the
    radix-shared pages count once. The append moves its rows twice (read, write)
    plus the slot mapping.
    """
    B, H, KVH, D = lay.batch, lay.num_heads, lay.num_kv_heads, lay.head_dim
    tokens = lay.unique_pages_tokens if (unique and lay.unique_pages is not None) else lay.kv_tokens()
    pages_used = int(((lay.context_lens.astype(np.int64) + lay.block_size - 1) // lay.block_size).sum())
    attn = tokens * KVH * D * 2 * elem_bytes + 2 * B * H * D * elem_bytes + pages_used * 4 + B * 4
    append = 2 * (2 * B * KVH * D * elem_bytes) + B * 8
    return dict(attention=attn, append=append, layer_call=attn + append)
