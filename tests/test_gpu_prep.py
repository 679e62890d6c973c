"""GPU parity of the pre-attention kernels (q/k RMSNorm + rotary embedding, the KV
write, and the one-launch norm + rotary + append + attention of a decode layer)
against the reference's golden outputs and the CPU oracle, through the C ABI.

Tolerances. Rotated q/k rows: within 2**-6 (bf16), 2**-9 (f16), 1e-6 (fp32)
of the largest magnitude of their head row against the reference's CPU outputs
(torch's CPU rsqrt rounds twice for 16-bit tensors), and within one unit in the
last place of that magnitude (fp32: eight) against the oracle, which rounds
where torch's CUDA kernels round. Attention outputs: the attention tolerances (bf16/f16 max
2e-2, mean 2e-3; fp32 max 1e-5). V rows and untouched pool slots: bit-exact.
"""
import numpy as np
import pytest
import torch

from conftest import PREP_GOLDEN_NAMES, load_prep_golden, sha

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ROW_TOL = {"bfloat16": 2.0 ** -6, "float16": 2.0 ** -9, "float32": 1e-6}
# against the oracle: one unit in the last place of the row's largest element for
# the 16-bit types; fp32 allows 8 (rsqrtf and the order of the sum of squares)
ULP = {"bfloat16": 2.0 ** -7, "float16": 2.0 ** -10, "float32": 2.0 ** -20}
ATT_TOL = {"float32": (1e-5, 1e-6), "bfloat16": (2e-2, 2e-3), "float16": (2e-2, 2e-3)}
TD = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def row_err(a: np.ndarray, ref: np.ndarray) -> float:
    scale = np.abs(ref).max(axis=-1, keepdims=True)
    return float((np.abs(a - ref) / np.maximum(scale, 1e-30)).max())


def f32(t):
    return t.float().cpu().numpy()


def dev(d):
    return {k: (v.to(DEV) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def golden_slots(z):
    if str(z["kind"]) == "decode":
        return torch.from_numpy(z["slot_mapping"])
    T, bs = int(z["num_tokens"]), int(z["block_size"])
    pos = z["positions"].astype(np.int64)
    return torch.from_numpy(z["block_table_row"][pos // bs].astype(np.int64) * bs + pos % bs)


def check_pool(z, caches, kc, vc, slots, k_ref, dtype):
    """V and untouched slots bit-exact; written K rows close to k_ref."""
    assert sha(vc.cpu()) == str(z["sha_v_after"])
    NB, bs = kc.shape[0], kc.shape[1]
    rows = f32(kc).reshape(NB * bs, -1)
    base = caches["k_cache"].float().numpy().reshape(NB * bs, -1)
    s = slots.numpy()
    written = np.zeros(NB * bs, dtype=bool)
    written[s] = True
    assert np.array_equal(rows[~written], base[~written])
    assert row_err(rows[s], k_ref.reshape(len(s), -1)) <= ROW_TOL[dtype]


@pytest.mark.parametrize("name", PREP_GOLDEN_NAMES)
def test_qk_norm_rope_golden(name, pkg, oracle):
    z, lay, x, caches, rope = load_prep_golden(name)
    dtype = str(z["dtype"])
    d, c = dev(x), dev(caches)
    slots = golden_slots(z)
    pos = torch.from_numpy(z["positions"]).to(DEV)
    q, k = pkg.qk_norm_rope(d["q_raw"], d["k_raw"], d["q_weight"], d["k_weight"], rope.to(DEV), pos,
                            float(z["eps"]), v=d["v_new"], k_cache=c["k_cache"], v_cache=c["v_cache"],
                            slot_mapping=slots.to(DEV))
    torch.cuda.synchronize()
    pkg.check_device_errors()
    qo, ko, _ = oracle.qk_norm_rope(x["q_raw"], x["k_raw"], x["q_weight"], x["k_weight"], rope, z["positions"],
                                    float(z["eps"]))
    for a, ref_g, ref_o in ((q, z["q_rot_ref"], qo), (k, z["k_rot_ref"], ko)):
        assert row_err(f32(a), ref_g) <= ROW_TOL[dtype]
        assert row_err(f32(a), ref_o) <= ULP[dtype]
    check_pool(z, caches, c["k_cache"], c["v_cache"], slots, z["k_rot_ref"], dtype)


@pytest.mark.parametrize("schedule", ["balanced", "split"])
@pytest.mark.parametrize("name", [n for n in PREP_GOLDEN_NAMES if "prefill" not in n])
def test_fused_prep_attention_golden(name, schedule, pkg):
    """Norm + rotary + append + attention in one launch against the reference's
    decode layer (engine.py:201-224)."""
    z, lay, x, caches, rope = load_prep_golden(name)
    dtype = str(z["dtype"])
    d, c = dev(x), dev(caches)
    out = pkg.paged_decode_prep_attention(
        d["q_raw"], d["k_raw"], d["v_new"], d["q_weight"], d["k_weight"], rope.to(DEV), c["k_cache"], c["v_cache"],
        torch.from_numpy(z["block_table"]).to(DEV), torch.from_numpy(z["context_lens"]).to(DEV), float(z["eps"]),
        schedule=schedule)
    torch.cuda.synchronize()
    pkg.check_device_errors()
    err = np.abs(f32(out).astype(np.float64) - z["out_ref"])
    mx, mean = ATT_TOL[dtype]
    assert err.max() <= mx and err.mean() <= mean, (err.max(), err.mean())
    check_pool(z, caches, c["k_cache"], c["v_cache"], golden_slots(z), z["k_rot_ref"], dtype)


def random_prep(pkg, seed, T, heads, dtype, positions_hi, with_pool=True):
    H, KVH, D = heads
    wl = pkg.workloads
    lay = wl.layout_uniform(seed, T, 1, positions_hi, num_heads=H, num_kv_heads=KVH, head_dim=D)
    caches = wl.materialize_host(lay, seed, dtype=dtype) if with_pool else None
    x = wl.materialize_prep_host(seed, T, H, KVH, D, dtype=dtype)
    rope = pkg.rope_table(D, positions_hi + 8, 500000.0)
    return lay, caches, x, rope


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("heads", [(16, 8, 112), (32, 8, 128), (16, 16, 64), (8, 2, 256), (4, 1, 80)])
def test_qk_norm_rope_random_vs_oracle(dtype, heads, pkg, oracle):
    seed = 300 + 3 * [(16, 8, 112), (32, 8, 128), (16, 16, 64), (8, 2, 256), (4, 1, 80)].index(heads) + \
        ["float32", "bfloat16", "float16"].index(dtype)
    lay, _, x, rope = random_prep(pkg, seed, 37, heads, dtype, 3000, with_pool=False)
    pos = lay.positions()
    d = dev(x)
    q, k = pkg.qk_norm_rope(d["q_raw"], d["k_raw"], d["q_weight"], d["k_weight"], rope.to(DEV),
                            torch.from_numpy(pos).to(DEV), 1e-6)
    qo, ko, _ = oracle.qk_norm_rope(x["q_raw"], x["k_raw"], x["q_weight"], x["k_weight"], rope, pos, 1e-6)
    for a, ref in ((q, qo), (k, ko)):
        e = row_err(f32(a), ref)
        assert e <= ULP[dtype], e
        if dtype != "float32":  # 16-bit: the same rounding points, so nearly all equal
            assert (f32(a) == ref).mean() >= 0.99


def test_qk_norm_rope_matches_torch_cuda_ops(pkg):
    """The kernel against the reference's RMSNorm and rotary formulas written as
    torch ops on the GPU (model.py:25-27 and :41-46; the engine runs them on
    CUDA), bf16: the same rounding points, so nearly every element is equal."""
    lay, _, x, rope = random_prep(pkg, 77, 64, (16, 8, 112), "bfloat16", 2048, with_pool=False)
    d = dev(x)
    pos = torch.from_numpy(lay.positions()).to(DEV)
    tab = rope.to(DEV)

    def ref_norm_rope(t, w):
        n = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6)
        n = n * w
        fc = torch.view_as_complex(tab[pos.long()].contiguous())          # (T, D/2)
        xc = torch.view_as_complex(n.float().reshape(*n.shape[:-1], -1, 2))
        return torch.view_as_real(xc * fc.unsqueeze(1)).flatten(2).type_as(t)

    q, k = pkg.qk_norm_rope(d["q_raw"], d["k_raw"], d["q_weight"], d["k_weight"], tab, pos, 1e-6)
    for a, r in ((q, ref_norm_rope(d["q_raw"], d["q_weight"])), (k, ref_norm_rope(d["k_raw"], d["k_weight"]))):
        assert row_err(f32(a), f32(r)) <= ULP["bfloat16"]
        assert (f32(a) == f32(r)).mean() >= 0.99


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("schedule", ["balanced", "split"])
def test_fused_prep_equals_two_launches(dtype, schedule, pkg):
    """One launch (norm + rotary + append + attention) against qk_norm_rope with
    the append followed by paged_attention on the same inputs."""
    seed = 400 + ["bfloat16", "float16", "float32"].index(dtype) * 2 + (schedule == "split")
    lay, caches, x, rope = random_prep(pkg, seed, 19, (16, 8, 112), dtype, 900)
    d, c1, c2 = dev(x), dev(caches), dev({k: v.clone() for k, v in caches.items()})
    bt, cl = c1["block_table"], c1["context_lens"]
    out1 = pkg.paged_decode_prep_attention(d["q_raw"], d["k_raw"], d["v_new"], d["q_weight"], d["k_weight"],
                                           rope.to(DEV), c1["k_cache"], c1["v_cache"], bt, cl, 1e-6,
                                           schedule=schedule)
    pos = cl - 1
    slots = pkg.slot_mapping(bt, pos, 16)
    q, _ = pkg.qk_norm_rope(d["q_raw"], d["k_raw"], d["q_weight"], d["k_weight"], rope.to(DEV), pos, 1e-6,
                            v=d["v_new"], k_cache=c2["k_cache"], v_cache=c2["v_cache"], slot_mapping=slots,
                            return_k=False)
    out2 = pkg.paged_attention(q, c2["k_cache"], c2["v_cache"], bt, cl, schedule=schedule)
    torch.cuda.synchronize()
    pkg.check_device_errors()
    assert torch.equal(c1["v_cache"], c2["v_cache"])
    # the two kernels sum the squares in different orders: the rotated rows may
    # differ by one unit in the last place, and the attention outputs by less
    # than the attention tolerance
    NB, bs = c1["k_cache"].shape[:2]
    k1 = f32(c1["k_cache"]).reshape(NB * bs, -1)
    k2 = f32(c2["k_cache"]).reshape(NB * bs, -1)
    assert row_err(k1, k2) <= ULP[dtype]
    err = np.abs(f32(out1) - f32(out2))
    mx, mean = ATT_TOL[dtype]
    assert err.max() <= mx and err.mean() <= mean


def test_bad_position_flagged_not_faulted(pkg):
    lay, caches, x, rope = random_prep(pkg, 91, 4, (16, 8, 112), "bfloat16", 100)
    d = dev(x)
    pos = torch.tensor([3, 5000, -1, 7], dtype=torch.int32, device=DEV)
    pkg.qk_norm_rope(d["q_raw"], d["k_raw"], d["q_weight"], d["k_weight"], rope.to(DEV), pos, 1e-6)
    with pytest.raises(RuntimeError, match="rotary position"):
        pkg.check_device_errors()
    # the fused kernel flags a context longer than the table
    c = dev(caches)
    short = rope[:10].to(DEV)
    pkg.paged_decode_prep_attention(d["q_raw"], d["k_raw"], d["v_new"], d["q_weight"], d["k_weight"], short,
                                    c["k_cache"], c["v_cache"], c["block_table"], c["context_lens"], 1e-6)
    with pytest.raises(RuntimeError, match="rotary position"):
        pkg.check_device_errors()


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_prefill_kv_write_bit_exact(dtype, pkg, oracle):
    """A prefill chunk's KV rows land where the reference's per-token write_kv
    loop (engine.py:126-128) puts them."""
    wl = pkg.workloads
    T, start, NB = 45, 21, 12
    lay = wl.Layout(np.array([start + T], dtype=np.int32), np.full((1, 6), -1, dtype=np.int32), NB)
    npages = (start + T + 15) // 16
    lay.block_table[0, :npages] = wl.portable_permutation(5, 2, NB)[:npages]
    caches = wl.materialize_host(lay, 5, dtype=dtype)
    x = wl.materialize_prep_host(5, T, 16, 8, 112, dtype=dtype)
    c = dev(caches)
    row = torch.from_numpy(lay.block_table[0]).to(DEV)
    slots = pkg.prefill_kv_write(x["k_raw"].to(DEV), x["v_new"].to(DEV), c["k_cache"], c["v_cache"], row, start)
    pos = np.arange(start, start + T, dtype=np.int32)
    ref_slots, st = oracle.slot_mapping(np.repeat(lay.block_table, T, 0), pos, 16)
    assert st == 0 and np.array_equal(slots.cpu().numpy(), ref_slots)
    kc, vc = caches["k_cache"].clone(), caches["v_cache"].clone()
    assert oracle.kv_append(x["k_raw"], x["v_new"], kc, vc, torch.from_numpy(ref_slots)) == 0
    torch.cuda.synchronize()
    assert torch.equal(c["k_cache"].cpu(), kc) and torch.equal(c["v_cache"].cpu(), vc)


def test_prefill_kv_write_edges(pkg, oracle):
    """The one-launch prefill write: a chunk that runs past its block-table row
    (no slot, nothing written), a -1 page inside the row (padding), K/V given as
    head-strided views (the copy path without contiguous head rows), and a page
    outside the pool (flagged, not written)."""
    T, start, NB, KVH, D = 50, 5, 10, 8, 112                     # positions 5 .. 54
    g = torch.Generator().manual_seed(31)
    kc = torch.randn((NB, 16, KVH, D), generator=g).to(torch.bfloat16)
    vc = torch.randn((NB, 16, KVH, D), generator=g).to(torch.bfloat16)
    big_k = torch.randn((T, KVH, 128), generator=g).to(torch.bfloat16)
    big_v = torch.randn((T, KVH, 128), generator=g).to(torch.bfloat16)
    k, v = big_k[:, :, :D], big_v[:, :, :D]                       # head stride 128, not D
    row = np.array([3, -1, 7], dtype=np.int32)                     # 3 pages: positions 0..47 only
    dkc, dvc = kc.to(DEV), vc.to(DEV)
    dk, dv = big_k.to(DEV)[:, :, :D], big_v.to(DEV)[:, :, :D]
    assert dk.stride(1) == 128
    slots = pkg.prefill_kv_write(dk, dv, dkc, dvc, torch.from_numpy(row).to(DEV), start)
    torch.cuda.synchronize()
    pos = np.arange(start, start + T)
    want = np.full(T, -1, dtype=np.int64)
    inside = pos // 16 < len(row)
    pages = np.where(inside, row[np.minimum(pos // 16, len(row) - 1)], -1)
    ok = inside & (pages >= 0)
    want[ok] = pages[ok] * 16 + pos[ok] % 16
    assert np.array_equal(slots.cpu().numpy(), want)
    ek, ev = kc.clone(), vc.clone()
    assert oracle.kv_append(k.contiguous(), v.contiguous(), ek, ev, torch.from_numpy(want)) == 0
    assert torch.equal(dkc.cpu(), ek) and torch.equal(dvc.cpu(), ev)
    pkg.check_device_errors()
    # a page id past the pool: reported, the pool left as it was
    bad = torch.tensor([NB + 2], dtype=torch.int32, device=DEV)
    before = dkc.clone()
    pkg.prefill_kv_write(dk[:4], dv[:4], dkc, dvc, bad, 0)
    torch.cuda.synchronize()
    assert torch.equal(dkc, before)
    with pytest.raises(RuntimeError, match="slot outside"):
        pkg.check_device_errors()


def test_prefill_prep_golden(pkg):
    z, lay, x, caches, rope = load_prep_golden("prep_prefill_fp32")
    d, c = dev(x), dev(caches)
    q, k = pkg.prefill_prep(d["q_raw"], d["k_raw"], d["v_new"], d["q_weight"], d["k_weight"], rope.to(DEV),
                            c["k_cache"], c["v_cache"], torch.from_numpy(z["block_table_row"]).to(DEV),
                            int(z["start_pos"]), float(z["eps"]))
    torch.cuda.synchronize()
    assert row_err(f32(q), z["q_rot_ref"]) <= ROW_TOL["float32"]
    assert row_err(f32(k), z["k_rot_ref"]) <= ROW_TOL["float32"]
    check_pool(z, caches, c["k_cache"], c["v_cache"], golden_slots(z), z["k_rot_ref"], "float32")


def test_prep_graph_capture(pkg):
    """The fused decode layer (norm + rotary + append + attention) replays from a
    CUDA graph with the same result as eager calls."""
    lay, caches, x, rope = random_prep(pkg, 55, 24, (16, 8, 112), "bfloat16", 700)
    d, c = dev(x), dev(caches)
    tab = rope.to(DEV)
    args = (d["q_raw"], d["k_raw"], d["v_new"], d["q_weight"], d["k_weight"], tab, c["k_cache"], c["v_cache"],
            c["block_table"], c["context_lens"], 1e-6)
    # both with programmatic overlap: the flag also shapes the work split (the last
    # CTA's range is shorter), so eager and replayed calls use the same one
    out_eager = pkg.paged_decode_prep_attention(*args, overlap_previous=True).clone()
    out = torch.empty_like(out_eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        pkg.paged_decode_prep_attention(*args, out=out, overlap_previous=True)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        pkg.paged_decode_prep_attention(*args, out=out, overlap_previous=True)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, out_eager)
