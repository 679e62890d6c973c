"""Generate the golden fixtures by running the reference's own CPU path.

Run in a container that has the reference checked out (read-only is fine):

    UNBOX_REFERENCE=<reference checkout> python tests/golden/make_golden.py

(or ``--reference <checkout>``).

The attention cases (CASES) cover the append and the attention call; the
pre-attention cases (PREP_CASES) add the q/k RMSNorm and rotary steps before
them. For each case it builds the inputs with the portable seeded generator
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


# Pre-attention cases: q_norm / k_norm (RMSNorm, unbox_platform/model/model.py:19-27),
# rotary embedding (model.py:30-48) and the KV write, run as the engine runs them
# (decode: engine.py:201-224 with positions = seq_lens - 1; prefill: engine.py:113-128).
# The model constants are those of ModelConfig (unbox_platform/model/config.py:25,28).
ROPE_THETA = 500000.0
RMS_EPS = 1e-6
PREP_CASES = {
    # name: (kind, spec, dtype, seed)
    "prep_attn_bf16": ("decode", dict(batch=6, ctx=(1, 200), num_blocks=128, heads=(16, 8, 112), rope_positions=208),
                       "bfloat16", 5),
    "prep_decode_f16_d64": ("decode", dict(batch=5, ctx=(1, 60), num_blocks=32, heads=(16, 4, 64),
                                           rope_positions=64), "float16", 6),
    "prep_prefill_fp32": ("prefill", dict(tokens=12, start=40, num_blocks=8, heads=(16, 8, 112), rope_positions=64),
                          "float32", 7),
}


def run_prep_case(ref_root, wl, name, kind, spec, dtype, seed):
    """Inputs from the portable generator; outputs from the reference's own
    RMSNorm / apply_rotary_emb / precompute_freqs_cis / PagedKVCache.write_kv /
    paged_decode_attention_ref, called the way the engine calls them. The rotary
    table is the complex64 freqs_cis of the model definition."""
    import torch
    sys.path.insert(0, ref_root)
    from unbox_platform.infer.kernels.paged_decode_attention import paged_decode_attention_ref
    from unbox_platform.infer.kvcache import PagedKVCache, SequenceState
    from unbox_platform.model.model import RMSNorm, apply_rotary_emb, precompute_freqs_cis

    td = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[dtype]
    H, KVH, D = spec["heads"]
    P = spec["rope_positions"]
    freqs_cis = precompute_freqs_cis(D, P, ROPE_THETA)
    if kind == "decode":
        lay = wl.layout_uniform(seed, spec["batch"], spec["ctx"][0], spec["ctx"][1], spec["num_blocks"],
                                num_heads=H, num_kv_heads=KVH, head_dim=D)
        T = lay.batch
        positions = (lay.context_lens.astype(np.int64) - 1)
        NB, bs = lay.num_blocks, lay.block_size
    else:
        T = spec["tokens"]
        positions = np.arange(spec["start"], spec["start"] + T, dtype=np.int64)
        NB, bs = spec["num_blocks"], 16
        lay = wl.Layout(np.array([spec["start"] + T], dtype=np.int32),
                        np.full((1, NB), -1, dtype=np.int32), NB, num_heads=H, num_kv_heads=KVH, head_dim=D)
        npages = (spec["start"] + T + bs - 1) // bs
        lay.block_table[0, :npages] = wl.portable_permutation(seed, 2, NB)[:npages]
    caches = wl.materialize_host(lay, seed, dtype=dtype)
    x = wl.materialize_prep_host(seed, T, H, KVH, D, dtype=dtype)

    q_norm, k_norm = RMSNorm(D, eps=RMS_EPS), RMSNorm(D, eps=RMS_EPS)
    with torch.no_grad():
        q_norm.weight.copy_(x["q_weight"].float())
        k_norm.weight.copy_(x["k_weight"].float())
    q_norm, k_norm = q_norm.to(td), k_norm.to(td)   # model.to(dtype), engine.py:84

    cache = PagedKVCache(num_layers=1, num_kv_heads=KVH, head_dim=D, num_blocks=NB, block_size=bs,
                         device=torch.device("cpu"), dtype=td)
    cache._pool.data[0, 0].copy_(caches["k_cache"])
    cache._pool.data[0, 1].copy_(caches["v_cache"])
    rec = {}
    with torch.no_grad():
        if kind == "decode":
            xq = q_norm(x["q_raw"].unsqueeze(1))      # (B, 1, H, D)
            xk = k_norm(x["k_raw"].unsqueeze(1))
            xv = x["v_new"].unsqueeze(1)
            for b in range(T):                         # engine.py:204-210
                pos = int(positions[b])
                fc = freqs_cis[pos: pos + 1]
                rq, rk = apply_rotary_emb(xq[b:b + 1], xk[b:b + 1], fc)
                xq[b:b + 1] = rq
                xk[b:b + 1] = rk
            seqs = []
            for b in range(T):
                n = int((lay.context_lens[b] + bs - 1) // bs)
                sq = SequenceState(request_id=f"r{b}", prompt_token_ids=list(range(int(lay.context_lens[b]))))
                sq.block_table = [int(v) for v in lay.block_table[b, :n]]
                seqs.append(sq)
            for b, sq in enumerate(seqs):             # engine.py:213-215
                cache.write_kv(0, sq, sq.total_len - 1, xk[b, 0], xv[b, 0])
            k_pool, v_pool = cache.get_kv_layer(0)
            q_for_kernel = xq[:, 0]
            if dtype != "float32":
                out = paged_decode_attention_ref(q_for_kernel.float(), k_pool.float(), v_pool.float(),
                                                 caches["block_table"], caches["context_lens"], bs)
            else:
                out = paged_decode_attention_ref(q_for_kernel, k_pool, v_pool, caches["block_table"],
                                                 caches["context_lens"], bs)
            rec.update(context_lens=lay.context_lens, block_table=lay.block_table, slot_mapping=lay.slot_mapping(),
                       out_ref=out.float().numpy())
            q_rot, k_rot = xq[:, 0], xk[:, 0]
        else:
            xq = q_norm(x["q_raw"].unsqueeze(0))      # (1, T, H, D), engine.py:121-123
            xk = k_norm(x["k_raw"].unsqueeze(0))
            xq, xk = apply_rotary_emb(xq, xk, freqs_cis[spec["start"]: spec["start"] + T])
            sq = SequenceState(request_id="p", prompt_token_ids=list(range(spec["start"] + T)))
            sq.block_table = [int(v) for v in lay.block_table[0] if v >= 0]
            for t in range(T):                         # engine.py:126-128
                cache.write_kv(0, sq, spec["start"] + t, xk[0, t], x["v_new"][t])
            k_pool, v_pool = cache.get_kv_layer(0)
            rec.update(block_table_row=lay.block_table[0], start_pos=np.array(spec["start"]))
            q_rot, k_rot = xq[0], xk[0]
    rec.update(
        name=np.array(name), kind=np.array(kind), dtype=np.array(dtype), seed=np.array(seed),
        num_heads=np.array(H), num_kv_heads=np.array(KVH), head_dim=np.array(D), block_size=np.array(bs),
        num_blocks=np.array(NB), num_tokens=np.array(T), eps=np.array(RMS_EPS), theta=np.array(ROPE_THETA),
        # only the table rows the tokens use (a kernel reads no other row)
        rope_positions=np.array(P), rope_rows=torch.view_as_real(freqs_cis).numpy()[positions].astype(np.float32),
        positions=positions.astype(np.int32),
        q_rot_ref=q_rot.float().numpy(), k_rot_ref=k_rot.float().numpy(),
        sha_q_raw=np.array(sha(x["q_raw"])), sha_k_raw=np.array(sha(x["k_raw"])), sha_v_new=np.array(sha(x["v_new"])),
        sha_q_weight=np.array(sha(x["q_weight"])), sha_k_weight=np.array(sha(x["k_weight"])),
        sha_k_cache=np.array(sha(caches["k_cache"])), sha_v_cache=np.array(sha(caches["v_cache"])),
        sha_k_after=np.array(sha(k_pool)), sha_v_after=np.array(sha(v_pool)),
    )
    return rec


# KV hand-off case: the reference's KVPool.serialize_blocks / deserialize_blocks
# (unbox_platform/infer/kvcache.py:268-277) on an fp32 pool, the only dtype its
# float32 payload decoding round-trips.
HANDOFF_CASES = {
    # name: (num_layers, num_blocks, num_kv_heads, head_dim, src pages, dst pages, seed)
    "handoff_fp32": (3, 12, 8, 112, [5, 0, 9, 3, 11], [7, 2, 11, 4, 0], 8),
}


def run_handoff_case(ref_root, wl, name, L, NB, KVH, D, src_pages, dst_pages, seed):
    import torch
    sys.path.insert(0, ref_root)
    from unbox_platform.infer.kvcache import KVPool

    src = KVPool(L, KVH, D, NB, 16, torch.device("cpu"), torch.float32)
    src.data.copy_(wl.materialize_pool_host(seed, L, NB, 16, KVH, D, "float32"))
    payload = src.serialize_blocks(src_pages)
    dst = KVPool(L, KVH, D, NB, 16, torch.device("cpu"), torch.float32)   # a fresh pool is zeros
    dst.deserialize_blocks(payload, dst_pages, (L, 2, len(dst_pages), 16, KVH, D))
    return dict(
        name=np.array(name), seed=np.array(seed), num_layers=np.array(L), num_blocks=np.array(NB),
        num_kv_heads=np.array(KVH), head_dim=np.array(D), block_size=np.array(16), dtype=np.array("float32"),
        src_pages=np.array(src_pages, dtype=np.int32), dst_pages=np.array(dst_pages, dtype=np.int32),
        sha_src_pool=np.array(sha(src.data)), payload_bytes=np.array(len(payload)),
        sha_payload=np.array(hashlib.sha256(payload).hexdigest()), sha_dst_after=np.array(sha(dst.data)),
    )


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("UNBOX_REFERENCE"),
                    help="reference checkout (default: $UNBOX_REFERENCE)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or UNBOX_REFERENCE")
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
    for name, (L, NB, KVH, D, sp, dp, seed) in HANDOFF_CASES.items():
        if args.only and name != args.only:
            continue
        rec = run_handoff_case(args.reference, wl, name, L, NB, KVH, D, sp, dp, seed)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **rec)
        print(f"{name}: {int(rec['payload_bytes'])} payload bytes -> {os.path.basename(path)}")
    for name, (kind, spec, dtype, seed) in PREP_CASES.items():
        if args.only and name != args.only:
            continue
        rec = run_prep_case(args.reference, wl, name, kind, spec, dtype, seed)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **rec)
        print(f"{name}: {kind} T={int(rec['num_tokens'])} -> {os.path.basename(path)}")


if __name__ == "__main__":
    main()
