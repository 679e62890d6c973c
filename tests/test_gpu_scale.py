"""GPU parity of the shapes and plans the multi-GPU and shared-prefix paths run.

* The KV-head slices that box-scale shards give each GPU for contexts over
  2048 tokens: (query heads, KV heads, head_dim) = (8, 4, 112), (4, 2, 112) and
  (2, 1, 112) at 2, 4 and 8 GPUs, against the oracle.
* The box-scale batch itself (1024 requests, log-normal contexts) cut by
  ``plan_shards`` for 1, 2, 4 and 8 GPUs: every shard is built from one global
  set of values (its own pages, permuted per rank, holding the global rows of
  its sequences and KV heads), run on cuda:0 in turn with the append fused, and
  reassembled. The reassembled output equals the single-call output within the
  attention tolerance and matches the oracle on sampled rows; every shard's
  pool equals the global pool after the append, bit for bit.
* The full-size radix-prefix batch (128 requests on 96 shared pages) through
  the plain kernel and through the cascade with the benchmark's own plan,
  every row against the oracle, the appended pools bit-exact.

Tolerances as in test_gpu_decode: bf16 attention max-abs 2e-2, mean-abs 2e-3
against the fp32/float64 reference on the same values; appends bit-exact.
Reference semantics: paged_decode_attention.py:157-191 (GQA map :168,175),
kvcache.py:253-262,330-340; the per-GPU split mirrors router.py:85-86 and
worker.py:47-51.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = {"float32": (1e-5, 1e-6), "bfloat16": (2e-2, 2e-3), "float16": (2e-2, 2e-3)}


def close(out, ref, dtype):
    err = np.abs(out.float().cpu().numpy().astype(np.float64) - ref)
    mx, mean = TOL[dtype]
    assert err.max() <= mx and err.mean() <= mean, (err.max(), err.mean())


def to_dev(t):
    return {k: v.to(DEV) for k, v in t.items()}


SLICES = [(8, 4, 112), (4, 2, 112), (2, 1, 112)]


@pytest.mark.parametrize("schedule", ["auto", "balanced", "split"])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("heads", SLICES)
def test_head_slice_shapes(heads, dtype, schedule, pkg, oracle):
    """One GPU's KV-head slice of long contexts: append fused, then attention."""
    H, KVH, D = heads
    wl = pkg.workloads
    seed = 300 + 7 * SLICES.index(heads) + {"bfloat16": 0, "float16": 1, "float32": 2}[dtype]
    lay = wl.layout_uniform(seed, 9, 1, 4200, num_heads=H, num_kv_heads=KVH, head_dim=D)
    t = wl.materialize_host(lay, seed, dtype=dtype, value_scale=0.7)
    d = to_dev(t)
    out = pkg.paged_attention(d["q"], d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"],
                              schedule=schedule, split_pages=7, k_new=d["k_new"], v_new=d["v_new"])
    torch.cuda.synchronize()
    pkg.check_device_errors()
    kc, vc = t["k_cache"].clone(), t["v_cache"].clone()
    assert oracle.kv_append(t["k_new"], t["v_new"], kc, vc, t["slot_mapping"]) == 0
    assert torch.equal(d["k_cache"].cpu(), kc) and torch.equal(d["v_cache"].cpu(), vc)
    ref, st = oracle.paged_decode_attention(t["q"], kc, vc, t["block_table"], t["context_lens"])
    assert st == 0
    close(out, ref, dtype)


# ---------------------------------------------------------------- box scale, sharded

def _page_pairs(glay, lay, seqs):
    """(global page, local page) of every (sequence, page index) of a shard part."""
    n = (lay.context_lens.astype(np.int64) + lay.block_size - 1) // lay.block_size
    w = lay.block_table.shape[1]
    mask = np.arange(w)[None, :] < n[:, None]
    gp = glay.block_table[seqs][:, :w][mask]
    lp = lay.block_table[mask]
    return torch.from_numpy(gp.astype(np.int64)).to(DEV), torch.from_numpy(lp.astype(np.int64)).to(DEV)


@pytest.fixture(scope="module")
def box_scale(pkg):
    """Global box-scale values (one layer) on cuda:0 and the single-call result."""
    wl = pkg.workloads
    glay = wl.named_layout("box_scale", seed=0)
    g = wl.materialize_device(glay, 17, "bfloat16", 1.0, 1, device=DEV)
    src = {"k": g["k_caches"][0].clone(), "v": g["v_caches"][0].clone()}  # before the append
    out = pkg.paged_attention(g["q"][0], g["k_caches"][0], g["v_caches"][0], g["block_table"], g["context_lens"],
                              k_new=g["k_new"][0], v_new=g["v_new"][0])
    torch.cuda.synchronize()
    pkg.check_device_errors()
    yield glay, g, src, out
    del g, src


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_box_scale_shards_reassemble(world, box_scale, pkg, oracle):
    glay, g, src, out_single = box_scale
    sh = pkg.sharding
    B, H, KVH, D = glay.batch, glay.num_heads, glay.num_kv_heads, glay.head_dim
    G = H // KVH
    shards = sh.plan_shards(glay.context_lens, world)
    sh.check_cover(shards, B, KVH)
    out = torch.full((B, H, D), float("nan"), dtype=torch.bfloat16, device=DEV)
    written = torch.zeros((B, H), dtype=torch.int32, device=DEV)
    for s in shards:
        parts = []
        if len(s.whole):
            parts.append((s.whole, 0, KVH, 1000 + s.rank))
        if s.kv_head_count:
            parts.append((s.head_split, s.kv_head_first, s.kv_head_count, 2000 + s.rank))
        for seqs, k0, nk, seed in parts:
            # the rank's own pool: its sequences' pages at a per-rank permutation, holding the
            # global rows of its KV heads (bench.py builds the same parts)
            lay = sh.local_layout(glay.context_lens, seqs, seed, G * nk, nk)
            gp, lp = _page_pairs(glay, lay, seqs)
            kc = torch.zeros((lay.num_blocks, 16, nk, D), dtype=torch.bfloat16, device=DEV)
            vc = torch.zeros_like(kc)
            kc[lp] = src["k"][gp][:, :, k0:k0 + nk]
            vc[lp] = src["v"][gp][:, :, k0:k0 + nk]
            si = torch.from_numpy(seqs.astype(np.int64)).to(DEV)
            q = g["q"][0][si][:, k0 * G:(k0 + nk) * G].contiguous()
            k_new = g["k_new"][0][si][:, k0:k0 + nk].contiguous()
            v_new = g["v_new"][0][si][:, k0:k0 + nk].contiguous()
            o = pkg.paged_attention(q, kc, vc, torch.from_numpy(lay.block_table).to(DEV),
                                    torch.from_numpy(lay.context_lens).to(DEV), k_new=k_new, v_new=v_new)
            torch.cuda.synchronize()
            pkg.check_device_errors()
            # the shard's pool after its append holds the global pool's bytes after the global append
            assert torch.equal(kc[lp], g["k_caches"][0][gp][:, :, k0:k0 + nk])
            assert torch.equal(vc[lp], g["v_caches"][0][gp][:, :, k0:k0 + nk])
            out[si.unsqueeze(1), torch.arange(k0 * G, (k0 + nk) * G, device=DEV).unsqueeze(0)] = o
            written[si.unsqueeze(1), torch.arange(k0 * G, (k0 + nk) * G, device=DEV).unsqueeze(0)] += 1
            del kc, vc
    assert torch.all(written == 1), "every (sequence, query head) comes from exactly one shard"
    diff = (out.float() - out_single.float()).abs()
    assert diff.max().item() <= 2e-2 and diff.mean().item() <= 2e-3, (diff.max().item(), diff.mean().item())
    # sampled rows against the oracle: the longest, the shortest and a spread of the rest,
    # with every head-split sequence's share represented
    order = np.argsort(glay.context_lens, kind="stable")
    rows = np.unique(np.concatenate([order[:4], order[-8:], order[:: max(1, B // 24)]]))
    bt = glay.block_table[rows]
    used = np.unique(bt[bt >= 0])
    remap = np.full(glay.num_blocks, -1, dtype=np.int64)
    remap[used] = np.arange(len(used))
    ui = torch.from_numpy(used.astype(np.int64)).to(DEV)
    kh, vh = g["k_caches"][0][ui].cpu(), g["v_caches"][0][ui].cpu()
    bt_sub = np.where(bt >= 0, remap[np.maximum(bt, 0)], -1).astype(np.int32)
    ref, st = oracle.paged_decode_attention(g["q"][0][torch.from_numpy(rows).to(DEV)].cpu(), kh, vh,
                                            torch.from_numpy(bt_sub), torch.from_numpy(glay.context_lens[rows]))
    assert st == 0
    close(out[torch.from_numpy(rows).to(DEV)], ref, "bfloat16")


# ---------------------------------------------------------------- radix prefix, full size

@pytest.mark.parametrize("path", ["plain", "cascade"])
def test_radix_prefix_full_size(path, pkg, oracle):
    """128 requests on 96 shared pages + private suffixes: the bench's exact inputs
    shape and plan; every row against the oracle, the append bit-exact."""
    wl = pkg.workloads
    lay = wl.named_layout("radix_prefix", seed=0)
    t = wl.materialize_host(lay, 19, dtype="bfloat16", value_scale=1.0)
    d = to_dev(t)
    if path == "plain":
        out = pkg.paged_attention(d["q"], d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"],
                                  k_new=d["k_new"], v_new=d["v_new"])
    else:
        plan = pkg.plan_cascade(lay.block_table, lay.context_lens, lay.num_heads, lay.num_kv_heads, device=DEV)
        assert plan.num_work > 0 and plan.shared_tokens == 96 * 16
        out = pkg.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], plan, k_new=d["k_new"],
                                          v_new=d["v_new"])
    torch.cuda.synchronize()
    pkg.check_device_errors()
    kc, vc = t["k_cache"].clone(), t["v_cache"].clone()
    assert oracle.kv_append(t["k_new"], t["v_new"], kc, vc, t["slot_mapping"]) == 0
    assert torch.equal(d["k_cache"].cpu(), kc) and torch.equal(d["v_cache"].cpu(), vc)
    ref, st = oracle.paged_decode_attention(t["q"], kc, vc, t["block_table"], t["context_lens"])
    assert st == 0
    close(out, ref, "bfloat16")
