"""GPU: shared-prefix (cascade) decode attention through the C ABI against the
reference's golden outputs and the oracle's attention over the original block
tables. Tolerances as for the attention kernel (bf16/f16 max-abs 2e-2,
mean-abs 2e-3 against an fp32 reference on the same values); the KV append is
bit-exact; the suffix pass's log-sum-exp within 1e-3 (log2 units) of float64."""
import numpy as np
import pytest
import torch

from conftest import load_golden, sha

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = (2e-2, 2e-3)


def close(out, ref):
    err = np.abs(out.float().cpu().numpy().astype(np.float64) - ref)
    assert err.max() <= TOL[0] and err.mean() <= TOL[1], (err.max(), err.mean())


def to_dev(t):
    return {k: v.to(DEV) for k, v in t.items()}


def test_cascade_golden_radix_with_append(pkg):
    """The reference's radix-shared case (12 requests on 6 shared pages, append
    of the decoded token, paged_decode_attention_ref)."""
    z, lay, t = load_golden("radix_small_bf16")
    d = to_dev(t)
    plan = pkg.plan_cascade(lay.block_table, lay.context_lens, lay.num_heads, lay.num_kv_heads,
                            min_shared_pages=2, device=DEV)
    assert plan.num_work > 0
    out = pkg.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], plan, k_new=d["k_new"],
                                      v_new=d["v_new"])
    torch.cuda.synchronize()
    pkg.check_device_errors()
    assert sha(d["k_cache"].cpu()) == str(z["sha_k_after"]) and sha(d["v_cache"].cpu()) == str(z["sha_v_after"])
    close(out, z["out_ref"].astype(np.float64))


CASES = [("bfloat16", (16, 8, 112)), ("float16", (16, 4, 64)), ("bfloat16", (32, 8, 128)),
         ("bfloat16", (16, 16, 64)), ("float16", (16, 2, 64)), ("bfloat16", (8, 8, 112))]


@pytest.mark.parametrize("schedule", ["balanced", "split"])
@pytest.mark.parametrize("dtype,heads", CASES)
def test_cascade_random_vs_oracle(dtype, heads, schedule, pkg, oracle):
    H, KVH, D = heads
    wl = pkg.workloads
    seed = 500 + 2 * CASES.index((dtype, heads)) + (schedule == "split")
    lay = wl.layout_radix_prefix(seed, batch=70, prefix_pages=21, suffix_lo=1, suffix_hi=300)
    lay.num_heads, lay.num_kv_heads, lay.head_dim = H, KVH, D
    t = wl.materialize_host(lay, seed, dtype=dtype, value_scale=0.7)
    d = to_dev(t)
    plan = pkg.plan_cascade(lay.block_table, lay.context_lens, H, KVH, device=DEV)
    assert plan.num_work > 0 and plan.max_chunks == -(-21 // pkg.cascade.MAX_CHUNK_PAGES)
    out = pkg.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], plan, schedule=schedule)
    ref, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"],
                                            t["context_lens"])
    assert st == 0
    torch.cuda.synchronize()
    pkg.check_device_errors()
    close(out, ref)


@pytest.mark.parametrize("prefix_ctas", [0, 1, 8, 40, 1000])
def test_cascade_one_launch_split_of_sms(prefix_ctas, pkg, oracle):
    """The suffix and prefix passes in one launch, with the SMs split between
    them in several ways (0: two launches; 1000: clamped to all CTAs but one,
    which then streams every suffix page), each with the append: the pools
    bit-exact against the oracle's write, the output within tolerance."""
    wl = pkg.workloads
    lay = wl.layout_radix_prefix(91, batch=96, prefix_pages=37, suffix_lo=1, suffix_hi=400)
    t = wl.materialize_host(lay, 91, dtype="bfloat16", value_scale=0.7)
    d = to_dev(t)
    plan = pkg.plan_cascade(lay.block_table, lay.context_lens, 16, 8, device=DEV)
    assert plan.num_work > 0 and plan.suffix_pages > 0
    out = pkg.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], plan, k_new=d["k_new"],
                                      v_new=d["v_new"], prefix_ctas=prefix_ctas)
    torch.cuda.synchronize()
    pkg.check_device_errors()
    kc, vc = t["k_cache"].clone(), t["v_cache"].clone()
    oracle.kv_append(t["k_new"], t["v_new"], kc, vc, t["slot_mapping"])
    assert torch.equal(d["k_cache"].cpu(), kc) and torch.equal(d["v_cache"].cpu(), vc)
    ref, st = oracle.paged_decode_attention(t["q"], kc, vc, t["block_table"], t["context_lens"])
    assert st == 0
    close(out, ref)


@pytest.mark.parametrize("prefix_ctas", [0, 20])
def test_members_with_empty_suffix(prefix_ctas, pkg, oracle):
    """Group members whose suffix is empty (their context ends with the shared
    pages): the result is their attention over the shared pages alone, and the
    suffix log-sum-exp reads -inf."""
    wl = pkg.workloads
    lay = wl.layout_radix_prefix(95, batch=40, prefix_pages=24, suffix_lo=1, suffix_hi=120)
    t = wl.materialize_host(lay, 95, dtype="bfloat16", value_scale=0.7)
    d = to_dev(t)
    plan = pkg.plan_cascade(lay.block_table, lay.context_lens, 16, 8, device=DEV)
    assert plan.num_work > 0
    members = sorted(b for mem, _ in plan.groups for b in mem)
    shared = {b: len(pages) for mem, pages in plan.groups for b in mem}
    empty = members[::3]
    sctx = plan.suffix_context_lens.cpu()
    ctx = t["context_lens"].clone()
    for b in empty:
        sctx[b] = 0
        ctx[b] = shared[b] * 16
    plan.suffix_context_lens = sctx.to(DEV)
    out = pkg.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], plan, prefix_ctas=prefix_ctas)
    torch.cuda.synchronize()
    pkg.check_device_errors()
    ref, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"], ctx)
    assert st == 0
    close(out, ref)
    lse = plan._lse.cpu()
    assert torch.isinf(lse[empty]).all() and (lse[empty] < 0).all()
    assert torch.isfinite(lse[[b for b in members if b not in empty]]).all()


@pytest.mark.parametrize("prefix_ctas", [0, 24])
def test_cascade_pool_with_interleaved_pages(prefix_ctas, pkg, oracle):
    """K and V pages interleaved in one allocation, (pages, 2, 16, KVH, D): the
    page stride is twice 16 token rows, so the shared pages are copied by
    address (page stride, token stride), not as one run of rows; with the
    append, pools bit-exact, output within tolerance."""
    wl = pkg.workloads
    lay = wl.layout_radix_prefix(97, batch=48, prefix_pages=26, suffix_lo=1, suffix_hi=200)
    t = wl.materialize_host(lay, 97, dtype="bfloat16", value_scale=0.7)
    d = to_dev(t)
    kv = torch.stack([d["k_cache"], d["v_cache"]], dim=1).contiguous()
    kc_dev, vc_dev = kv[:, 0], kv[:, 1]
    assert kc_dev.stride(0) == 2 * kc_dev.stride(1) * kc_dev.shape[1]
    plan = pkg.plan_cascade(lay.block_table, lay.context_lens, 16, 8, device=DEV)
    assert plan.num_work > 0
    out = pkg.paged_attention_cascade(d["q"], kc_dev, vc_dev, plan, k_new=d["k_new"], v_new=d["v_new"],
                                      prefix_ctas=prefix_ctas)
    torch.cuda.synchronize()
    pkg.check_device_errors()
    kc, vc = t["k_cache"].clone(), t["v_cache"].clone()
    oracle.kv_append(t["k_new"], t["v_new"], kc, vc, t["slot_mapping"])
    assert torch.equal(kc_dev.cpu(), kc) and torch.equal(vc_dev.cpu(), vc)
    ref, st = oracle.paged_decode_attention(t["q"], kc, vc, t["block_table"], t["context_lens"])
    assert st == 0
    close(out, ref)


def test_cascade_two_groups_and_unshared_requests(pkg, oracle):
    """Two prefix groups side by side with requests that share nothing: the
    unshared ones go through the suffix pass alone."""
    wl = pkg.workloads
    a = wl.layout_radix_prefix(61, batch=10, prefix_pages=9, suffix_lo=1, suffix_hi=90)
    b = wl.layout_radix_prefix(62, batch=7, prefix_pages=13, suffix_lo=30, suffix_hi=60)
    u = wl.layout_uniform(63, 5, 1, 200, num_blocks=80)
    mb = max(a.block_table.shape[1], b.block_table.shape[1], u.block_table.shape[1])
    bts, ctxs, off = [], [], 0
    for lay in (a, b, u):
        bt = np.full((lay.batch, mb), -1, dtype=np.int32)
        bt[:, :lay.block_table.shape[1]] = np.where(lay.block_table >= 0, lay.block_table + off, -1)
        bts.append(bt)
        ctxs.append(lay.context_lens)
        off += lay.num_blocks
    lay = wl.Layout(np.concatenate(ctxs), np.concatenate(bts), off)
    t = wl.materialize_host(lay, 64, dtype="bfloat16")
    d = to_dev(t)
    plan = pkg.plan_cascade(lay.block_table, lay.context_lens, 16, 8, device=DEV)
    assert len(plan.groups) == 2
    out = pkg.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], plan)
    ref, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"],
                                            t["context_lens"])
    torch.cuda.synchronize()
    close(out, ref)


def test_suffix_lse_matches_float64(pkg):
    """ubx_paged_decode_attention_lse's log-sum-exp (log2 units, scores scaled by
    scale * log2 e) against float64, balanced and split schedules."""
    wl = pkg.workloads
    lay = wl.layout_uniform(71, 6, 1, 700)
    t = wl.materialize_host(lay, 71, dtype="bfloat16")
    d = to_dev(t)
    plan = pkg.plan_cascade(lay.block_table, lay.context_lens, 16, 8, device=DEV)   # no groups
    q, kc = t["q"].double().numpy(), t["k_cache"].double().numpy()
    scale = 112 ** -0.5
    want = np.zeros((6, 16))
    for b in range(6):
        n = int(lay.context_lens[b])
        rows = np.concatenate([kc[p] for p in lay.block_table[b, :(n + 15) // 16]], axis=0)[:n]
        for h in range(16):
            s = rows[:, h // 2] @ q[b, h] * scale * np.log2(np.e)
            want[b, h] = s.max() + np.log2(np.exp2(s - s.max()).sum())
    for schedule in ("balanced", "split"):
        pkg.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], plan, schedule=schedule)
        torch.cuda.synchronize()
        assert np.abs(plan._lse.cpu().numpy() - want).max() < 1e-3


def test_cascade_graph_capture_and_fp32_refused(pkg):
    wl = pkg.workloads
    lay = wl.layout_radix_prefix(81, batch=24, prefix_pages=16, suffix_lo=1, suffix_hi=100)
    t = wl.materialize_host(lay, 81, dtype="bfloat16")
    d = to_dev(t)
    plan = pkg.plan_cascade(lay.block_table, lay.context_lens, 16, 8, device=DEV)
    eager = pkg.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], plan).clone()
    out = torch.empty_like(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        pkg.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], plan, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        pkg.paged_attention_cascade(d["q"], d["k_cache"], d["v_cache"], plan, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    with pytest.raises(TypeError):
        pkg.paged_attention_cascade(d["q"].float(), d["k_cache"].float(), d["v_cache"].float(), plan)
