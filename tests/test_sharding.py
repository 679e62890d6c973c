"""CPU: multi-GPU partitioning of a decode batch (host logic), and a two-rank
gloo run in which each rank attends only to its shard and the gathered result
equals the single-process result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG


def test_lpt_balances_loads():
    sh = PKG.sharding
    rng = np.random.default_rng(0)
    costs = rng.integers(1, 1000, size=300)
    bins = sh.lpt(costs, 8)
    loads = [costs[b].sum() for b in bins]
    assert sorted(i for b in bins for i in b) == list(range(300))
    assert max(loads) - min(loads) <= costs.max()


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_box_scale_plan_covers_every_head_once(world):
    sh, wl = PKG.sharding, PKG.workloads
    lay = wl.named_layout("box_scale")
    shards = sh.plan_shards(lay.context_lens, world)
    sh.check_cover(shards, lay.batch, 8)
    kv = [s.kv_bytes for s in shards]
    total = int(lay.context_lens.astype(np.int64).sum()) * 8 * 112 * 2 * 2
    assert sum(kv) == total
    if world > 1:
        # long contexts are head-split, the rest LPT-placed: loads within one request's bytes
        assert max(kv) - min(kv) <= int(lay.context_lens.max()) * 8 * 112 * 2 * 2
        assert all(len(s.head_split) == int((lay.context_lens > 2048).sum()) for s in shards)


def test_head_split_disabled_when_heads_do_not_divide():
    sh = PKG.sharding
    ctx = np.array([5000, 100, 200])
    shards = sh.plan_shards(ctx, 3, num_kv_heads=8)
    assert all(s.kv_head_count == 0 for s in shards)
    sh.check_cover(shards, 3, 8)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from __graft_entry__ import load_package
        from oracle import oracle
        pkg = load_package()
        wl = pkg.workloads
        lay = wl.layout_uniform(50, 10, 1, 300)
        t = wl.materialize_host(lay, 50, dtype="float32")
        shards = pkg.sharding.plan_shards(lay.context_lens, world, long_threshold=200)
        mine = shards[rank]
        G = lay.num_heads // lay.num_kv_heads
        part = {}
        if len(mine.whole):
            w = torch.from_numpy(mine.whole)
            out, st = oracle.paged_decode_attention(t["q"][w], t["k_cache"], t["v_cache"], t["block_table"][w],
                                                    t["context_lens"][w])
            part["whole"] = (mine.whole, out)
        if mine.kv_head_count:
            hs = torch.from_numpy(mine.head_split)
            k0, kc = mine.kv_head_first, mine.kv_head_count
            q = t["q"][hs][:, k0 * G:(k0 + kc) * G]
            out, st = oracle.paged_decode_attention(q, t["k_cache"][:, :, k0:k0 + kc], t["v_cache"][:, :, k0:k0 + kc],
                                                    t["block_table"][hs], t["context_lens"][hs])
            part["heads"] = (mine.head_split, k0 * G, (k0 + kc) * G, out)
        gathered = [None] * world
        dist.all_gather_object(gathered, part)
        if rank == 0:
            full = np.zeros((lay.batch, lay.num_heads, lay.head_dim))
            seen = np.zeros((lay.batch, lay.num_heads), dtype=int)
            for g in gathered:
                if "whole" in g:
                    idx, out = g["whole"]
                    full[idx] = out
                    seen[idx] += 1
                if "heads" in g:
                    idx, h0, h1, out = g["heads"]
                    full[idx, h0:h1] = out
                    seen[idx, h0:h1] += 1
            ref, _ = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"],
                                                   t["context_lens"])
            np.savez(out_path, full=full, ref=ref, seen=seen, long=int((lay.context_lens > 200).sum()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reassemble_the_batch(tmp_path):
    port = _free_port()
    out = str(tmp_path / "res.npz")
    mp.start_processes(_rank_main, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    r = np.load(out)
    assert r["long"] > 0, "the case must exercise the KV-head split"
    assert np.all(r["seen"] == 1)
    assert np.array_equal(r["full"], r["ref"])
