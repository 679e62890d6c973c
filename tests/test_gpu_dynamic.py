"""GPU: the dynamic (work-sharing) schedule of the decode kernel against the
reference's golden outputs and the oracle, through the C ABI. Same tolerances
as the other schedules (bf16/f16 max-abs 2e-2, mean-abs 2e-3 against an fp32
reference on the same values; the KV append bit-exact). The schedule re-arms its
workspace words at the end of every launch, so most tests call it repeatedly,
with different batches, and interleave it with the balanced schedule."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN_NAMES, load_golden, sha

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = (2e-2, 2e-3)


def close(out, ref):
    err = np.abs(out.float().cpu().numpy().astype(np.float64) - ref)
    assert err.max() <= TOL[0] and err.mean() <= TOL[1], (err.max(), err.mean())


def to_dev(t):
    return {k: v.to(DEV) for k, v in t.items()}


@pytest.mark.parametrize("name", [n for n in GOLDEN_NAMES if "fp32" not in n])
def test_dynamic_golden_with_fused_append(name, pkg):
    z, lay, t = load_golden(name)
    d = to_dev(t)
    out = pkg.paged_attention(d["q"], d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"],
                              lay.head_dim ** -0.5, schedule="dynamic", k_new=d["k_new"], v_new=d["v_new"])
    torch.cuda.synchronize()
    pkg.check_device_errors()
    assert sha(d["k_cache"].cpu()) == str(z["sha_k_after"]) and sha(d["v_cache"].cpu()) == str(z["sha_v_after"])
    close(out, z["out_ref"].astype(np.float64))


CASES = [("bfloat16", (16, 8, 112)), ("float16", (16, 8, 112)), ("bfloat16", (16, 16, 64)),
         ("bfloat16", (32, 8, 128)), ("float16", (16, 2, 64)), ("bfloat16", (8, 8, 112)), ("bfloat16", (8, 1, 128))]


@pytest.mark.parametrize("dtype,heads", CASES)
def test_dynamic_random_vs_oracle_repeated(dtype, heads, pkg, oracle):
    H, KVH, D = heads
    wl = pkg.workloads
    seed = 600 + CASES.index((dtype, heads))
    lay = wl.layout_uniform(seed, 23, 1, 900, num_heads=H, num_kv_heads=KVH, head_dim=D)
    t = wl.materialize_host(lay, seed, dtype=dtype, value_scale=0.7)
    d = to_dev(t)
    ref, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"],
                                            t["context_lens"], 0.3)
    assert st == 0
    for sched in ("dynamic", "dynamic", "balanced", "dynamic"):
        out = pkg.paged_attention(d["q"], d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"], 0.3,
                                  schedule=sched)
        torch.cuda.synchronize()
        close(out, ref)
    pkg.check_device_errors()


@pytest.mark.parametrize("shape", ["one_long", "tiny", "mixed_zero", "box"])
def test_dynamic_shapes(shape, pkg, oracle):
    """One sequence over every CTA; fewer pages than CTAs; empty contexts mixed
    in; a 512-request log-normal batch, more requests than CTAs (sampled rows)."""
    wl = pkg.workloads
    if shape == "one_long":
        lay = wl.layout_uniform(71, 1, 30000, 30001)
    elif shape == "tiny":
        lay = wl.layout_uniform(72, 40, 1, 20)
    elif shape == "mixed_zero":
        lay = wl.layout_uniform(73, 30, 1, 400)
        lay.context_lens[::4] = 0
    else:
        lay = wl.layout_lognormal(74, batch=512, median=96.0, lo=16, hi=384)
    t = wl.materialize_host(lay, 75, dtype="bfloat16")
    d = to_dev(t)
    out = pkg.paged_attention(d["q"], d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"],
                              schedule="dynamic")
    bal = pkg.paged_attention(d["q"], d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"],
                              schedule="balanced")
    torch.cuda.synchronize()
    pkg.check_device_errors()
    if shape == "box":
        rows = np.arange(0, 512, 19)
        ref, st = oracle.paged_decode_attention(t["q"][rows], t["k_cache"], t["v_cache"], t["block_table"][rows],
                                                t["context_lens"][rows])
        close(out[rows], ref)
    else:
        ref, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"],
                                                t["context_lens"])
        close(out, ref)
    assert (st == 0) or shape == "mixed_zero"
    # the two schedules split the sums differently: equal to the attention tolerance
    err = (out.float() - bal.float()).abs()
    assert err.max().item() <= TOL[0]


def test_dynamic_batches_back_to_back_and_fused_prep(pkg, oracle):
    """Launches of different grids on one workspace, then the one-launch norm +
    rotary + append + attention under the dynamic schedule."""
    wl = pkg.workloads
    for i, (b, lo, hi) in enumerate([(64, 100, 600), (3, 1, 40), (200, 10, 300), (64, 100, 600)]):
        lay = wl.layout_uniform(80 + i, b, lo, hi)
        t = wl.materialize_host(lay, 80 + i, dtype="bfloat16", value_scale=0.5)
        d = to_dev(t)
        out = pkg.paged_attention(d["q"], d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"],
                                  schedule="dynamic", k_new=d["k_new"], v_new=d["v_new"])
        kc, vc = t["k_cache"].clone(), t["v_cache"].clone()
        assert oracle.kv_append(t["k_new"], t["v_new"], kc, vc, t["slot_mapping"]) == 0
        ref, _ = oracle.paged_decode_attention(t["q"], kc, vc, t["block_table"], t["context_lens"])
        torch.cuda.synchronize()
        assert torch.equal(d["k_cache"].cpu(), kc) and torch.equal(d["v_cache"].cpu(), vc)
        close(out, ref)
    # fused pre-attention through the dynamic schedule equals the balanced one
    lay = wl.layout_uniform(90, 19, 1, 900)
    caches = wl.materialize_host(lay, 90, dtype="bfloat16")
    x = wl.materialize_prep_host(90, 19, 16, 8, 112, dtype="bfloat16")
    rope = pkg.rope_table(112, 1024).to(DEV)
    outs = []
    for sched in ("balanced", "dynamic"):
        c = to_dev(caches)
        dx = to_dev(x)
        outs.append((pkg.paged_decode_prep_attention(dx["q_raw"], dx["k_raw"], dx["v_new"], dx["q_weight"],
                                                     dx["k_weight"], rope, c["k_cache"], c["v_cache"],
                                                     c["block_table"], c["context_lens"], schedule=sched), c))
    torch.cuda.synchronize()
    pkg.check_device_errors()
    (o1, c1), (o2, c2) = outs
    assert torch.equal(c1["k_cache"], c2["k_cache"]) and torch.equal(c1["v_cache"], c2["v_cache"])
    assert (o1.float() - o2.float()).abs().max().item() <= TOL[0]


def test_dynamic_graph_layers_with_overlap(pkg, oracle):
    """Six layer-calls with programmatic overlap, captured in a CUDA graph and
    replayed twice: every layer equals the oracle."""
    wl = pkg.workloads
    lay = wl.layout_uniform(95, 32, 100, 1200)
    L = 6
    ts = [wl.materialize_host(lay, 95 + l, dtype="bfloat16", value_scale=0.5) for l in range(L)]
    ds = [to_dev(t) for t in ts]
    outs = [torch.empty_like(d["q"]) for d in ds]

    def step():
        for d, o in zip(ds, outs):
            pkg.paged_attention(d["q"], d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"], out=o,
                                schedule="dynamic", overlap_previous=False)

    step()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for d, o in zip(ds, outs):
            pkg.paged_attention(d["q"], d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"], out=o,
                                schedule="dynamic", k_new=d["k_new"], v_new=d["v_new"], overlap_previous=True)
    for _ in range(2):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for t, o in zip(ts, outs):
            kc, vc = t["k_cache"].clone(), t["v_cache"].clone()
            oracle.kv_append(t["k_new"], t["v_new"], kc, vc, t["slot_mapping"])
            ref, _ = oracle.paged_decode_attention(t["q"], kc, vc, t["block_table"], t["context_lens"])
            close(o, ref)
    pkg.check_device_errors()


def test_dynamic_refuses_fp32_and_strided_new_rows(pkg):
    wl = pkg.workloads
    lay = wl.layout_uniform(97, 4, 1, 100)
    t = to_dev(wl.materialize_host(lay, 97, dtype="float32"))
    with pytest.raises(ValueError, match="dynamic"):
        pkg.paged_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"], t["context_lens"],
                            schedule="dynamic")
    tb = to_dev(wl.materialize_host(lay, 97, dtype="bfloat16"))
    kn = torch.zeros((4, 8, 128), dtype=torch.bfloat16, device=DEV)[:, :, :112]   # head stride 128
    with pytest.raises(ValueError, match="contiguous"):
        pkg.paged_attention(tb["q"], tb["k_cache"], tb["v_cache"], tb["block_table"], tb["context_lens"],
                            schedule="dynamic", k_new=kn, v_new=kn)
