import glob
import hashlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")
sys.path.insert(0, ROOT)

from __graft_entry__ import load_package  # noqa: E402

PKG = load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def sha(t) -> str:
    import torch
    x = t.contiguous()
    if x.dtype == torch.bfloat16:
        x = x.view(torch.int16)
    return hashlib.sha256(x.numpy().tobytes()).hexdigest()


_ALL_GOLDEN = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))
GOLDEN_NAMES = [n for n in _ALL_GOLDEN if not n.startswith(("prep_", "handoff_", "engine_"))]  # append + attention
PREP_GOLDEN_NAMES = [n for n in _ALL_GOLDEN if n.startswith("prep_")]  # norm + rotary (+ append, attention)
HANDOFF_GOLDEN_NAMES = [n for n in _ALL_GOLDEN if n.startswith("handoff_")]  # serialize / deserialize
ENGINE_GOLDEN_NAMES = [n for n in _ALL_GOLDEN if n.startswith("engine_")]  # the engine's decode flow


def load_engine_golden(name: str):
    """Engine-flow fixture (tests/golden/make_engine_golden.py): the record and
    the KV pool as prefill left it, (L, 2, NB, bs, KVH, D) in the case's dtype
    (checked by SHA-256)."""
    import torch
    z = dict(np.load(os.path.join(GOLDEN_DIR, name + ".npz")))
    td = {"float32": torch.float32, "bfloat16": torch.bfloat16}[str(z["dtype"])]
    pool0 = torch.from_numpy(z["pool0"]).to(td)
    assert sha(pool0) == str(z["sha_pool0"]), f"{name}: stored pool differs from the engine's"
    return z, pool0


def engine_block_table(blocks_of_step) -> "np.ndarray":
    """The decode step's block table as engine.py:179-185 builds it: int32,
    (batch, longest block list), padded with -1."""
    rows = [[int(x) for x in r if x >= 0] for r in blocks_of_step]
    bt = np.full((len(rows), max(len(r) for r in rows)), -1, dtype=np.int32)
    for i, r in enumerate(rows):
        bt[i, :len(r)] = r
    return bt


def load_golden(name: str):
    """Fixture record, its layout and the regenerated host inputs (checked by SHA-256)."""
    z = dict(np.load(os.path.join(GOLDEN_DIR, name + ".npz")))
    wl = PKG.workloads
    lay = wl.Layout(z["context_lens"], z["block_table"], int(z["num_blocks"]), int(z["num_heads"]),
                    int(z["num_kv_heads"]), int(z["head_dim"]), int(z["block_size"]))
    if "unique_pages" in z:
        lay.unique_pages = int(z["unique_pages"])
        lay.unique_pages_tokens = int(z["unique_pages_tokens"])
    t = wl.materialize_host(lay, int(z["seed"]), dtype=str(z["dtype"]), value_scale=float(z["value_scale"]))
    for k in ("q", "k_cache", "v_cache", "k_new", "v_new"):
        assert sha(t[k]) == str(z["sha_" + k]), f"{name}: regenerated {k} differs from the fixture's inputs"
    assert np.array_equal(t["slot_mapping"].numpy(), z["slot_mapping"])
    return z, lay, t


def load_prep_golden(name: str):
    """Pre-attention fixture: the record, the regenerated inputs (checked by
    SHA-256), the pool before the write, the layout and a rotary table of
    ``rope_positions`` rows holding the reference's rows at the used positions
    (the other rows are zero and never read)."""
    import torch
    z = dict(np.load(os.path.join(GOLDEN_DIR, name + ".npz")))
    wl = PKG.workloads
    H, KVH, D = int(z["num_heads"]), int(z["num_kv_heads"]), int(z["head_dim"])
    T, dtype, seed = int(z["num_tokens"]), str(z["dtype"]), int(z["seed"])
    if str(z["kind"]) == "decode":
        lay = wl.Layout(z["context_lens"], z["block_table"], int(z["num_blocks"]), H, KVH, D, int(z["block_size"]))
    else:
        start = int(z["start_pos"])
        lay = wl.Layout(np.array([start + T], dtype=np.int32), z["block_table_row"][None, :].copy(),
                        int(z["num_blocks"]), H, KVH, D, int(z["block_size"]))
    caches = wl.materialize_host(lay, seed, dtype=dtype)
    x = wl.materialize_prep_host(seed, T, H, KVH, D, dtype=dtype)
    for k in ("q_raw", "k_raw", "v_new", "q_weight", "k_weight"):
        assert sha(x[k]) == str(z["sha_" + k]), f"{name}: regenerated {k} differs from the fixture's inputs"
    for k in ("k_cache", "v_cache"):
        assert sha(caches[k]) == str(z["sha_" + k]), f"{name}: regenerated {k} differs"
    rope = np.zeros((int(z["rope_positions"]), D // 2, 2), dtype=np.float32)
    rope[z["positions"]] = z["rope_rows"]
    return z, lay, x, caches, torch.from_numpy(rope)


@pytest.fixture(scope="session")
def pkg():
    return PKG


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.build()
    return o
