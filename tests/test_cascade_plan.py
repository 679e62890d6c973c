"""CPU: the shared-prefix (cascade) planner (unbox_b200.cascade.plan_cascade).

The plan must split every grouped request's context exactly into the group's
shared pages and the request's own suffix, so that the log-sum-exp merge of the
two attentions equals attention over the whole context. Checked with a float64
numpy attention over the plan's pieces against the oracle's full attention.
"""
import numpy as np
import pytest

from conftest import PKG


def plan(lay, **kw):
    return PKG.cascade.plan_cascade(lay.block_table, lay.context_lens, lay.num_heads, lay.num_kv_heads,
                                    device="cpu", **kw)


def attend(q, k_cache, v_cache, pages, ntok, scale):
    """(H, D) attention of one request over the first ntok tokens of `pages`;
    returns (out (H, D), lse (H,)) in float64, natural log."""
    H, D = q.shape
    KVH = k_cache.shape[2]
    G = H // KVH
    rows_k = np.concatenate([k_cache[p] for p in pages], axis=0)[:ntok]   # (ntok, KVH, D)
    rows_v = np.concatenate([v_cache[p] for p in pages], axis=0)[:ntok]
    out = np.zeros((H, D))
    lse = np.full(H, -np.inf)
    if ntok == 0:
        return out, lse
    for h in range(H):
        s = rows_k[:, h // G] @ q[h] * scale
        m = s.max()
        w = np.exp(s - m)
        out[h] = w @ rows_v[:, h // G] / w.sum()
        lse[h] = m + np.log(w.sum())
    return out, lse


def merge(parts):
    M = max(l.max() for _, l in parts)
    num = sum(o * np.exp(l - M)[:, None] for o, l in parts)
    den = sum(np.exp(l - M) for _, l in parts)
    return num / den[:, None]


def test_radix_layout_groups_and_suffix_tables():
    wl = PKG.workloads
    lay = wl.layout_radix_prefix(3, batch=20, prefix_pages=12, suffix_lo=1, suffix_hi=70)
    p = plan(lay)
    assert len(p.groups) == 1
    members, shared = p.groups[0]
    assert sorted(members) == list(range(20)) and len(shared) == 12
    assert shared == lay.block_table[0, :12].tolist()
    assert p.max_chunks == 2
    sbt, sctx = p.suffix_block_table.numpy(), p.suffix_context_lens.numpy()
    for b in range(20):
        assert sctx[b] == lay.context_lens[b] - 12 * 16 >= 1
        n = (sctx[b] + 15) // 16
        assert np.array_equal(sbt[b, :n], lay.block_table[b, 12:12 + n])
    # every (member, chunk) pair covered by exactly one work item
    seen = {}
    mlist = p.member_list.numpy()
    for m_off, nm, pg_off, npg, chunk, _ in p.work.numpy():
        assert 1 <= npg <= PKG.cascade.MAX_CHUNK_PAGES and nm * 2 <= 128
        for b in mlist[m_off:m_off + nm]:
            seen[(int(b), int(chunk))] = seen.get((int(b), int(chunk)), 0) + 1
    assert set(seen.values()) == {1} and len(seen) == 20 * 2
    assert sorted(map(tuple, p.merge_items.numpy().tolist())) == [(b, 2) for b in range(20)]


def test_no_sharing_and_short_prefixes_stay_plain():
    wl = PKG.workloads
    lay = wl.layout_uniform(4, 9, 20, 300, num_blocks=200)
    p = plan(lay)
    assert p.num_work == 0 and p.num_merge == 0
    assert np.array_equal(p.suffix_block_table.numpy(), lay.block_table)
    # a shared prefix shorter than min_shared_pages is left alone
    lay2 = wl.layout_radix_prefix(5, batch=6, prefix_pages=3, suffix_lo=1, suffix_hi=30)
    assert plan(lay2, min_shared_pages=4).num_work == 0
    assert plan(lay2, min_shared_pages=2).num_work > 0


def test_prefix_cut_leaves_every_member_a_private_token():
    """A member whose context ends inside (or at the end of) the shared pages
    caps the group's prefix: the token being decoded stays on a private page."""
    wl = PKG.workloads
    lay = wl.layout_radix_prefix(6, batch=5, prefix_pages=10, suffix_lo=5, suffix_hi=40)
    lay.context_lens[2] = 6 * 16          # ends exactly at the end of page 5
    p = plan(lay)
    members, shared = p.groups[0]
    assert len(shared) == 5               # (96 - 1) // 16
    assert p.suffix_context_lens.numpy()[2] == 16


def test_prefix_cut_before_another_requests_append_page():
    """A shared page that also holds another request's append slot (a table no
    radix cache makes) is left out of the prefix: the shared pages are read while
    the suffix pass appends."""
    wl = PKG.workloads
    lay = wl.layout_radix_prefix(7, batch=5, prefix_pages=10, suffix_lo=5, suffix_hi=40)
    shared_page = int(lay.block_table[0, 7])
    outsider = wl.layout_uniform(8, 1, 40, 41, num_blocks=lay.num_blocks)
    bt = np.full((6, lay.block_table.shape[1]), -1, dtype=np.int32)
    bt[:5] = lay.block_table
    bt[5, :3] = [int(outsider.block_table[0, 0]), int(outsider.block_table[0, 1]), shared_page]
    ctx = np.concatenate([lay.context_lens, [40]]).astype(np.int32)   # position 39 lies on page index 2
    lay2 = wl.Layout(ctx, bt, lay.num_blocks)
    members, shared = plan(lay2).groups[0]
    assert len(shared) == 7 and shared_page not in shared


@pytest.mark.parametrize("heads", [(16, 8), (16, 2), (8, 8)])
def test_member_blocks_fill_one_tensor_core_tile(heads):
    """A large group is cut into member blocks of at most 128 / G members (one
    128-row tile of (request, query head) rows per work item); every member of
    every chunk is covered once, and the merge items list the members in
    member-list order with the group's chunk count."""
    H, KVH = heads
    G = H // KVH
    wl = PKG.workloads
    lay = wl.layout_radix_prefix(9, batch=150, prefix_pages=19, suffix_lo=1, suffix_hi=40)
    p = PKG.cascade.plan_cascade(lay.block_table, lay.context_lens, H, KVH, device="cpu")
    cap = PKG.cascade.TILE_ROWS // G
    nch = -(-19 // PKG.cascade.MAX_CHUNK_PAGES)
    work = p.work.numpy()
    assert (work[:, 1] <= cap).all() and (work[:, 3] <= PKG.cascade.MAX_CHUNK_PAGES).all()
    assert len(work) == nch * -(-150 // cap)
    cover = {}
    mlist = p.member_list.numpy()
    for m_off, nm, _, _, chunk, _ in work:
        for b in mlist[m_off:m_off + nm]:
            cover[(int(b), int(chunk))] = cover.get((int(b), int(chunk)), 0) + 1
    assert set(cover.values()) == {1} and len(cover) == 150 * nch
    items = p.merge_items.numpy()
    assert np.array_equal(items[:, 0], mlist) and (items[:, 1] == nch).all()


@pytest.mark.parametrize("heads", [(16, 8, 112), (16, 2, 64), (8, 8, 64)])
def test_merge_of_plan_pieces_equals_full_attention(heads, oracle):
    """Attention over the suffix table + attention over the shared pages, merged
    by log-sum-exp, equals the oracle's attention over the original table."""
    H, KVH, D = heads
    wl = PKG.workloads
    lay = wl.layout_radix_prefix(7, batch=9, prefix_pages=9, suffix_lo=1, suffix_hi=50)
    lay.num_heads, lay.num_kv_heads, lay.head_dim = H, KVH, D
    t = wl.materialize_host(lay, 7, dtype="float32")
    p = plan(lay)
    full, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"],
                                             t["context_lens"])
    assert st == 0
    q, kc, vc = (t[k].numpy().astype(np.float64) for k in ("q", "k_cache", "v_cache"))
    scale = D ** -0.5
    members, shared = p.groups[0]
    sbt, sctx = p.suffix_block_table.numpy(), p.suffix_context_lens.numpy()
    for b in members:
        n = (sctx[b] + 15) // 16
        o_s, l_s = attend(q[b], kc, vc, sbt[b, :n], int(sctx[b]), scale)
        o_p, l_p = attend(q[b], kc, vc, shared, len(shared) * 16, scale)
        np.testing.assert_allclose(merge([(o_s, l_s), (o_p, l_p)]), full[b], atol=1e-9)


@pytest.mark.parametrize("max_parts,run_pages", [(4, 24), (2, 48), (12, 8), (1, 64)])
def test_long_prefix_in_runs_of_chunks(max_parts, run_pages):
    """A 96-page shared prefix is cut into at most max_parts runs of whole 8-page
    chunks, each at most 64 pages (one work item per run and member block,
    folded on the device a chunk at a time); every (member, run) is covered once
    and the runs tile the shared pages in order."""
    wl = PKG.workloads
    lay = wl.layout_radix_prefix(11, batch=40, prefix_pages=96, suffix_lo=1, suffix_hi=60)
    p = PKG.cascade.plan_cascade(lay.block_table, lay.context_lens, 16, 8, max_parts=max_parts, device="cpu")
    n_runs = -(-96 // run_pages)
    assert p.max_chunks == n_runs
    work = p.work.numpy()
    assert (work[:, 3] <= min(run_pages, PKG.cascade.MAX_ITEM_PAGES)).all()
    starts = sorted({(int(w[4]), int(w[2]), int(w[3])) for w in work})
    assert [s[0] for s in starts] == list(range(n_runs))
    assert starts[0][1] == 0 and all(a[1] + a[2] == b[1] for a, b in zip(starts, starts[1:]))
    assert starts[-1][1] + starts[-1][2] == 96
    cover = {}
    mlist = p.member_list.numpy()
    for m_off, nm, _, _, part, _ in work:
        for b in mlist[m_off:m_off + nm]:
            cover[(int(b), int(part))] = cover.get((int(b), int(part)), 0) + 1
    assert set(cover.values()) == {1} and len(cover) == 40 * n_runs
    assert (p.merge_items.numpy()[:, 1] == n_runs).all()
