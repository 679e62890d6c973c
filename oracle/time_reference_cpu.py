"""Time the reference's own CPU path for one decode layer-call. Test and
CPU-baseline infrastructure only (nothing in the library imports it).

The reference's only working decode-attention path is the Python
``paged_decode_attention_ref`` (unbox_platform/infer/kernels/
paged_decode_attention.py:157-191, a loop over sequence, head and position),
preceded by the engine's per-sequence ``PagedKVCache.write_kv``
(unbox_platform/infer/kvcache.py:330-340, engine.py:213-215). It is far too
slow to run a whole layer-call of the benchmark workloads, so this script runs
it unmodified on a fixed seeded subsample -- a few sequences of the workload,
all heads, one layer -- and extrapolates linearly per (sequence, head,
position), which is how its cost grows. The reference checkout is needed, so
this runs where the reference is importable (not on the GPU hosts); its output,
``oracle/reference_cpu_path.json``, records the host, the core count torch used
and the sample, and bench.py reports it beside the oracle's own CPU timing,
labelled as extrapolated.

    UNBOX_REFERENCE=<reference checkout> python oracle/time_reference_cpu.py
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "reference_cpu_path.json")

# workload -> (layout seed the benchmark's rank 0 uses, sequences in the sample)
WORKLOADS = {"decode_760m": (1000, 3), "box_scale": (0, 3), "radix_prefix": (1000, 2), "long_context": (1000, 1)}


def host_info():
    model = None
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_count": os.cpu_count(), "usable_cpus": len(os.sched_getaffinity(0)), "cpu_model": model}


def time_workload(ref_root, name, seed, n_sample):
    import torch
    sys.path.insert(0, ref_root)
    sys.path.insert(0, ROOT)
    from unbox_platform.infer.kernels.paged_decode_attention import paged_decode_attention_ref
    from unbox_platform.infer.kvcache import PagedKVCache, SequenceState
    from __graft_entry__ import load_package

    wl = load_package().workloads
    lay = wl.named_layout(name, seed=seed)
    H, KVH, D, bs = lay.num_heads, lay.num_kv_heads, lay.head_dim, lay.block_size
    # the sample: sequences at evenly spaced ranks of the context length (shortest .. longest)
    order = np.argsort(lay.context_lens, kind="stable")
    rows = order[np.linspace(0, lay.batch - 1, n_sample).round().astype(int)]
    ctx = lay.context_lens[rows].astype(np.int64)
    npg = (ctx + bs - 1) // bs
    g = torch.Generator().manual_seed(5)
    nb = int(npg.sum())
    cache = PagedKVCache(num_layers=1, num_kv_heads=KVH, head_dim=D, num_blocks=nb, block_size=bs,
                         device=torch.device("cpu"), dtype=torch.bfloat16)
    cache._pool.data.copy_(torch.randn(cache._pool.data.shape, generator=g).to(torch.bfloat16))
    seqs, cur = [], 0
    bt = torch.full((len(rows), int(npg.max())), -1, dtype=torch.int32)
    for i, c in enumerate(ctx):
        s = SequenceState(request_id=f"r{i}", prompt_token_ids=list(range(int(c))))
        s.block_table = list(range(cur, cur + int(npg[i])))
        bt[i, :npg[i]] = torch.tensor(s.block_table, dtype=torch.int32)
        cur += int(npg[i])
        seqs.append(s)
    q = torch.randn((len(rows), H, D), generator=g).to(torch.bfloat16)
    k_new = torch.randn((len(rows), KVH, D), generator=g).to(torch.bfloat16)
    v_new = torch.randn((len(rows), KVH, D), generator=g).to(torch.bfloat16)
    seq_lens = torch.from_numpy(ctx.astype(np.int32))
    t0 = time.perf_counter()
    for i, s in enumerate(seqs):                       # engine.py:213-215
        cache.write_kv(0, s, s.total_len - 1, k_new[i], v_new[i])
    t_append = time.perf_counter() - t0
    k_pool, v_pool = cache.get_kv_layer(0)
    t0 = time.perf_counter()
    paged_decode_attention_ref(q, k_pool, v_pool, bt, seq_lens, bs)   # engine.py:221-224
    t_attn = time.perf_counter() - t0
    bhp = float(ctx.sum()) * H                           # (sequence, head, position) triples sampled
    per_bhp = t_attn / bhp
    per_seq_append = t_append / len(rows)
    full_bhp = float(lay.context_lens.astype(np.int64).sum()) * H
    t_call = per_bhp * full_bhp + per_seq_append * lay.batch
    ab = wl.algorithmic_bytes(lay, 2)["layer_call"]
    return {
        "workload": name, "layout_seed": seed, "dtype": "bf16",
        "sample": {"sequences": [int(r) for r in rows], "context_lens": [int(c) for c in ctx], "heads": H,
                   "layer": 0, "attention_s": round(t_attn, 4), "append_s": round(t_append, 5)},
        "per_seq_head_pos_us": round(per_bhp * 1e6, 3), "append_per_seq_us": round(per_seq_append * 1e6, 2),
        "extrapolated_layer_call_s": round(t_call, 3), "layer_call_bytes": int(ab),
        "value": round(ab / t_call / 1e9, 6), "unit": "GB/s", "layer_calls_per_s": round(1.0 / t_call, 6),
        "torch_threads": torch.get_num_threads(),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("UNBOX_REFERENCE"),
                    help="reference checkout (default: $UNBOX_REFERENCE)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or UNBOX_REFERENCE")
    rec = {"kind": "reference", "extrapolated": True, "path": "paged_decode_attention_ref + PagedKVCache.write_kv",
           "when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()), **host_info(), "workloads": {}}
    for name, (seed, n) in WORKLOADS.items():
        if args.only and name != args.only:
            continue
        r = time_workload(args.reference, name, seed, n)
        rec["workloads"][name] = r
        print(f"{name}: {r['per_seq_head_pos_us']} us per (seq, head, pos) -> {r['extrapolated_layer_call_s']} s "
              f"per layer-call, {r['value']} GB/s")
    with open(OUT, "w") as f:
        json.dump(rec, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
