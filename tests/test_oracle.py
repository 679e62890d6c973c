"""CPU: the oracle is pinned to the reference's own outputs (golden fixtures),
and, where the reference checkout is present, to the reference run live."""
import os
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN_NAMES, load_golden, sha

# checkout of the reference project (read-only is fine); the live test skips without it
REFERENCE = os.environ.get("UNBOX_REFERENCE", "")


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_oracle_matches_reference_golden(name, oracle):
    z, lay, t = load_golden(name)
    kc, vc = t["k_cache"].clone(), t["v_cache"].clone()
    assert oracle.kv_append(t["k_new"], t["v_new"], kc, vc, t["slot_mapping"]) == 0
    # the append is a byte copy: identical to the reference's PagedKVCache.write_kv result
    assert sha(kc) == str(z["sha_k_after"]) and sha(vc) == str(z["sha_v_after"])
    out, st = oracle.paged_decode_attention(t["q"], kc, vc, t["block_table"], t["context_lens"])
    assert st == 0
    err = np.abs(out - z["out_ref"])
    # the reference runs fp32 torch arithmetic; the oracle sums in double
    assert err.max() <= 1e-5, err.max()
    assert err.mean() <= 1e-6, err.mean()


def test_oracle_single_thread_equals_threaded(oracle):
    z, lay, t = load_golden("correctness_fp32")
    a, _ = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"], t["context_lens"],
                                         nthreads=1)
    b, _ = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"], t["context_lens"],
                                         nthreads=4)
    assert np.array_equal(a, b)


def test_oracle_uses_every_core_on_request(oracle):
    """The CPU baseline asks for every core the process may use, whatever
    OMP_NUM_THREADS said (torchrun sets it to 1 for its ranks)."""
    oracle.lib().oracle_set_num_threads(1)
    assert oracle.num_threads() == 1
    n = len(os.sched_getaffinity(0))
    assert oracle.use_all_cores() == n == oracle.num_threads()


def test_oracle_status_codes(oracle, pkg):
    lay = pkg.workloads.layout_uniform(5, 3, 1, 40, num_blocks=16)
    t = pkg.workloads.materialize_host(lay, 5)
    cl = t["context_lens"].clone()
    cl[1] = 0
    out, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"], cl)
    assert st == 1 and np.all(out[1] == 0)  # the reference raises on an empty context
    bt = t["block_table"].clone()
    bt[0, 0] = 10_000
    _, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], bt, t["context_lens"])
    assert st == 2
    cl = t["context_lens"].clone()
    cl[2] = 16 * bt.shape[1] + 1
    _, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"], cl)
    assert st == 4


def test_oracle_negative_page_wraps_like_python(oracle, pkg):
    """paged_decode_attention_ref indexes k_pool[-1] for a -1 entry (Python indexing)."""
    lay = pkg.workloads.layout_uniform(6, 2, 17, 30, num_blocks=8)
    t = pkg.workloads.materialize_host(lay, 6)
    bt = t["block_table"].clone()
    bt[0, 1] = -1
    bt2 = t["block_table"].clone()
    bt2[0, 1] = lay.num_blocks - 1
    a, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], bt, t["context_lens"])
    b, st2 = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], bt2, t["context_lens"])
    assert st == 0 and st2 == 0 and np.array_equal(a, b)


def test_slot_mapping_oracle(oracle, pkg):
    lay = pkg.workloads.named_layout("decode_760m")
    sm, st = oracle.slot_mapping(lay.block_table, lay.positions(), lay.block_size)
    assert st == 0 and np.array_equal(sm, lay.slot_mapping())


def test_portable_generator_is_stable(pkg):
    wl = pkg.workloads
    a = wl.portable_normal(0, 10, 5)
    # pinned values: the golden fixtures depend on this stream
    assert np.allclose(a, wl.portable_normal(0, 10, 5))
    assert np.all(np.abs(a * 65536 - np.round(a * 65536)) == 0)
    lay = wl.named_layout("correctness")
    assert lay.batch == 8 and lay.context_lens.min() >= 64 and lay.context_lens.max() <= 512
    assert lay.num_blocks == 512
    used = lay.block_table[lay.block_table >= 0]
    assert len(np.unique(used)) == len(used)


@pytest.mark.skipif(not REFERENCE or not os.path.isdir(os.path.join(REFERENCE, "unbox_platform")),
                    reason="UNBOX_REFERENCE does not name a reference checkout")
def test_oracle_against_live_reference(oracle, pkg):
    """Runs the reference's paged_decode_attention_ref itself on a fresh seed."""
    sys.path.insert(0, REFERENCE)
    from unbox_platform.infer.kernels.paged_decode_attention import paged_decode_attention_ref
    lay = pkg.workloads.layout_uniform(11, 3, 1, 90, num_blocks=40)
    t = pkg.workloads.materialize_host(lay, 11)
    ref = paged_decode_attention_ref(t["q"], t["k_cache"], t["v_cache"], t["block_table"], t["context_lens"], 16)
    out, st = oracle.paged_decode_attention(t["q"], t["k_cache"], t["v_cache"], t["block_table"], t["context_lens"])
    assert st == 0
    assert np.abs(out - ref.numpy()).max() <= 1e-5
