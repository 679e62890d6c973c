"""Generate the golden fixtures by running the reference's own CPU path.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py --reference /root/reference

For each case it builds the inputs with the portable seeded generator
(``workloads.materialize_host``), then runs, unmodified, the reference's
``PagedKVCache.write_kv`` (unbox_platform/infer/kvcache.py:330-340) for the new
token of every sequence and ``paged_decode_attention_ref``
(unbox_platform/infer/kernels/paged_decode_attention.py:157-191) over the
appended cache. It stores the seeds, the layout, a SHA-256 of every generated
input and the reference outputs, so the tests can regenerate the inputs
anywhere, prove they are the same bytes, and compare against what the
reference computed. bf16 cases run the reference in fp32 on the bf16 values
(upcast), the comparison the attention tolerance is defined against; the append
always runs in the case's own dtype because it is a byte copy.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from __graft_entry__ import load_package  # noqa: E402

CASES = {
    # name: (layout spec, dtype, value_scale, seed)
    "correctness_fp32": (dict(kind="uniform", batch=8, ctx=(64, 512), num_blocks=512), "float32", 1.0, 0),
    "small_bf16": (dict(kind="uniform", batch=6, ctx=(1, 200), num_blocks=128), "bfloat16", 0.5, 1),
    "edge_fp32": (dict(kind="edge"), "float32", 1.0, 2),
    "radix_small_bf16": (dict(kind="radix", batch=12, prefix_pages=6, suffix=(1, 70)), "bfloat16", 1.0, 3),
    "gqa4_d64_fp16": (dict(kind="uniform", batch=5, ctx=(1, 90), num_blocks=64, heads=(16, 4, 64)), "float16", 1.0, 4),
}


def sha(t) -> str:
    import torch
    x = t.contiguous()
    if x.dtype == torch.bfloat16:
        x = x.view(torch.int16)
    return hashlib.sha256(x.numpy().tobytes()).hexdigest()


def build_layout(wl, spec, seed):
    if spec["kind"] == "uniform":
        h = spec.get("heads", (16, 8, 112))
        return wl.layout_uniform(seed, spec["batch"], spec["ctx"][0], spec["ctx"][1], spec["num_blocks"],
                                 num_heads=h[0], num_kv_heads=h[1], head_dim=h[2])
    if spec["kind"] == "radix":
        return wl.layout_radix_prefix(seed, batch=spec["batch"], prefix_pages=spec["prefix_pages"],
                                      suffix_lo=spec["suffix"][0], suffix_hi=spec["suffix"][1])
    return edge_layout(wl, seed)


def edge_layout(wl, seed):
    """Edge cases in one batch: ctx 1, exact page multiples (16, 32), one token
    past a page boundary (17), a full 16-page row, a long-ish row, and a row
    whose table has extra -1 padding beyond what it needs."""
    ctx = np.array([1, 16, 17, 32, 256, 255, 2, 100], dtype=np.int32)
    nb = 96
    perm = wl.portable_permutation(seed, 2, nb)
    pages = (ctx + 15) // 16
    bt = np.full((ctx.shape[0], 20), -1, dtype=np.int32)
    cur = 0
    for b in range(ctx.shape[0]):
        bt[b, :pages[b]] = perm[cur:cur + pages[b]]
        cur += int(pages[b])
    return wl.Layout(ctx, bt, nb)


def run_reference(ref_root, lay, t, dtype):
    import torch
    sys.path.insert(0, ref_root)
    from unbox_platform.infer.kernels.paged_decode_attention import paged_decode_attention_ref
    from unbox_platform.infer.kvcache import PagedKVCache, SequenceState

    td = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[dtype]
    cache = PagedKVCache(num_layers=1, num_kv_heads=lay.num_kv_heads, head_dim=lay.head_dim,
                         num_blocks=lay.num_blocks, block_size=lay.block_size,
                         device=torch.device("cpu"), dtype=td)
    cache._pool.data[0, 0].copy_(t["k_cache"])
    cache._pool.data[0, 1].copy_(t["v_cache"])
    seqs = []
    for b in range(lay.batch):
        n = int((lay.context_lens[b] + lay.block_size - 1) // lay.block_size)
        s = SequenceState(request_id=f"r{b}", prompt_token_ids=list(range(int(lay.context_lens[b]))))
        s.block_table = [int(x) for x in lay.block_table[b, :n]]
        seqs.append(s)
    # the engine's append loop (engine.py:213-215): token at total_len - 1
    for b, s in enumerate(seqs):
        cache.write_kv(0, s, s.total_len - 1, t["k_new"][b], t["v_new"][b])
    k_pool, v_pool = cache.get_kv_layer(0)
    q = t["q"]
    if dtype != "float32":   # fp32 reference on the low-precision values
        qf, kf, vf = q.float(), k_pool.float(), v_pool.float()
    else:
        qf, kf, vf = q, k_pool, v_pool
    t0 = time.time()
    out = paged_decode_attention_ref(qf, kf, vf, t["block_table"], t["context_lens"], lay.block_size)
    el = time.time() - t0
    return k_pool.clone(), v_pool.clone(), out, el


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    pkg = load_package()
    wl = pkg.workloads
    for name, (spec, dtype, vs, seed) in CASES.items():
        if args.only and name != args.only:
            continue
        lay = build_layout(wl, spec, seed)
        t = wl.materialize_host(lay, seed, dtype=dtype, value_scale=vs)
        k_after, v_after, out, el = run_reference(args.reference, lay, t, dtype)
        rec = dict(
            name=np.array(name), dtype=np.array(dtype), seed=np.array(seed), value_scale=np.array(vs),
            num_heads=np.array(lay.num_heads), num_kv_heads=np.array(lay.num_kv_heads),
            head_dim=np.array(lay.head_dim), block_size=np.array(lay.block_size),
            num_blocks=np.array(lay.num_blocks),
            context_lens=lay.context_lens, block_table=lay.block_table,
            slot_mapping=lay.slot_mapping(),
            out_ref=out.float().numpy(),
            sha_q=np.array(sha(t["q"])), sha_k_cache=np.array(sha(t["k_cache"])),
            sha_v_cache=np.array(sha(t["v_cache"])), sha_k_new=np.array(sha(t["k_new"])),
            sha_v_new=np.array(sha(t["v_new"])),
            sha_k_after=np.array(sha(k_after)), sha_v_after=np.array(sha(v_after)),
            ref_seconds=np.array(el),
        )
        if lay.unique_pages is not None:
            rec["unique_pages"] = np.array(lay.unique_pages)
            rec["unique_pages_tokens"] = np.array(lay.unique_pages_tokens)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **rec)
        print(f"{name}: B={lay.batch} sum_ctx={lay.kv_tokens()} ref {el:.2f}s -> {os.path.basename(path)}")


if __name__ == "__main__":
    main()
