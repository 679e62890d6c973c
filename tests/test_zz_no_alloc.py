"""GPU: the allocation-free attention entry point agrees with the workspace one.

ubx_paged_decode_attention_noalloc serves callers that cannot allocate device
memory (an engine that hands all free HBM to its own KV pool, or a binding from
another language that holds only input and output buffers): its scratch is a
fixed array inside the library. This file is collected last on purpose, so that
a failure here comes after every other test has already run; it also passes on
its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def call_noalloc(lib, d, out, err, schedule=0, split_pages=0, max_blocks=None, batch=None):
    q, kc, vc, bt, cl = d["q"], d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"]
    B, H, D = q.shape
    NB, bs, KVH, _ = kc.shape
    return lib.ubx_paged_decode_attention_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1),
        kc.stride(2), bt.data_ptr(), bt.stride(0), cl.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
        B if batch is None else batch, H, KVH, D, bs, NB, bt.shape[1] if max_blocks is None else max_blocks,
        D ** -0.5, 1, schedule, split_pages, err.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point_twice(pkg):
    lib = pkg.library.load()
    wl = pkg.workloads
    lay = wl.layout_uniform(41, 48, 1, 2500)
    host = wl.materialize_host(lay, 41, dtype="bfloat16", value_scale=0.5)
    d = {k: v.to(DEV) for k, v in host.items()}
    q2 = (torch.randn(d["q"].shape, generator=torch.Generator().manual_seed(5)) * 0.5).to(torch.bfloat16).to(DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    outs = []
    for q in (d["q"], q2):   # two calls in a row, different queries, same shared scratch
        dq = dict(d, q=q)
        out = torch.empty_like(q)
        st = call_noalloc(lib, dq, out, err)
        assert st == 0, lib.ubx_last_error()
        outs.append(out)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for q, out in zip((d["q"], q2), outs):
        ref = pkg.paged_attention(q, d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"])
        e = (out.float() - ref.float()).abs()
        assert e.max().item() <= 2e-2 and e.mean().item() <= 2e-3


def test_noalloc_rejects_sizes_beyond_its_scratch(pkg):
    lib = pkg.library.load()
    wl = pkg.workloads
    lay = wl.layout_uniform(42, 4, 1, 64)
    d = {k: v.to(DEV) for k, v in wl.materialize_host(lay, 42, dtype="bfloat16").items()}
    out = torch.empty_like(d["q"])
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    # split schedule with one page per chunk and a huge (claimed) table width: the
    # partials would need far more than the fixed array; rejected before any launch
    st = call_noalloc(lib, d, out, err, schedule=2, split_pages=1, max_blocks=1 << 20)
    assert st == pkg.library.ERR_WORKSPACE
    assert b"fixed" in lib.ubx_last_error() and b"8388608" in lib.ubx_last_error()


@pytest.mark.parametrize("schedule,heads", [(1, (16, 8, 112)), (2, (16, 8, 112)), (2, (4, 4, 64))])
def test_noalloc_balanced_and_split_schedules_twice(schedule, heads, pkg, oracle):
    """The balanced schedule (merge counters, partials of cut sequences) and the
    split one (partials + log-sum-exp combine) keep all their scratch in the
    fixed array; the second call runs on what the first one left there."""
    lib = pkg.library.load()
    wl = pkg.workloads
    H, KVH, D = heads
    lay = wl.layout_uniform(43 + schedule, 48, 1, 2500, num_heads=H, num_kv_heads=KVH, head_dim=D)
    host = wl.materialize_host(lay, 43 + schedule, dtype="bfloat16", value_scale=0.5)
    d = {k: v.to(DEV) for k, v in host.items()}
    g = torch.Generator().manual_seed(6)
    q2_host = (torch.randn(host["q"].shape, generator=g) * 0.5).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    name = {1: "balanced", 2: "split"}[schedule]
    for q_host in (host["q"], q2_host):
        q = q_host.to(DEV)
        out = torch.empty_like(q)
        st = call_noalloc(lib, dict(d, q=q), out, err, schedule=schedule, split_pages=32)
        assert st == 0, lib.ubx_last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        ref = pkg.paged_attention(q, d["k_cache"], d["v_cache"], d["block_table"], d["context_lens"],
                                  schedule=name, split_pages=32)
        e = (out.float() - ref.float()).abs()
        assert e.max().item() <= 2e-2 and e.mean().item() <= 2e-3
        exact, _ = oracle.paged_decode_attention(q_host, host["k_cache"], host["v_cache"], host["block_table"],
                                                 host["context_lens"])
        e = np.abs(out.float().cpu().numpy().astype(np.float64) - exact)
        assert e.max() <= 2e-2 and e.mean() <= 2e-3
