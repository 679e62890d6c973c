"""CPU: the oracle replays the reference engine's decode flow and reproduces it.

The fixtures (tests/golden/make_engine_golden.py) record three decode steps of
the reference ``InferenceEngine.decode_step`` (engine.py:157-234) over a small
random model (head_dim 112, 4 query heads on 2 KV heads, 3 layers). Replaying
them here with the oracle checks the fixtures themselves and the flow the GPU
test (test_gpu_engine_flow.py) drives through the kernels: the block table and
lengths built as at engine.py:179-185, the append of every sequence's token at
total_len - 1 (:213-215) into the layer's pool, then attention over total_len
positions (:221-224); a later step's context includes the tokens earlier steps
appended.
"""
import numpy as np
import pytest
import torch

from conftest import ENGINE_GOLDEN_NAMES, engine_block_table, load_engine_golden, sha


def test_engine_fixtures_present():
    assert set(ENGINE_GOLDEN_NAMES) >= {"engine_decode_fp32", "engine_decode_bf16"}


@pytest.mark.parametrize("name", ENGINE_GOLDEN_NAMES)
def test_oracle_replays_engine_decode(name, oracle):
    z, pool = load_engine_golden(name)
    td = pool.dtype
    L, S = int(z["num_layers"]), int(z["steps"])
    for s in range(S):
        bt = engine_block_table(z["blocks"][s])
        rec = z["block_table_rec"][s][:, :bt.shape[1]]
        assert np.array_equal(bt, rec), "block table as engine.py:179-185 builds it"
        total = z["total"][s].astype(np.int32)
        assert np.array_equal(total, z["seq_lens_rec"][s])
        slots, st = oracle.slot_mapping(bt, total - 1, 16)
        assert st == 0
        for l in range(L):
            kp, vp = pool[l, 0], pool[l, 1]
            k_rows = torch.from_numpy(z["k_rows"][s, l]).to(td)
            v_rows = torch.from_numpy(z["v_rows"][s, l]).to(td)
            assert oracle.kv_append(k_rows, v_rows, kp, vp, torch.from_numpy(slots)) == 0
            assert sha(kp) == str(z["sha_k_after"][s, l]) and sha(vp) == str(z["sha_v_after"][s, l])
            q = torch.from_numpy(z["q"][s, l]).to(td)
            out, st = oracle.paged_decode_attention(q, kp, vp, torch.from_numpy(bt), torch.from_numpy(total))
            assert st == 0
            err = np.abs(out - z["out_ref32"][s, l])
            assert err.max() <= 1e-5, err.max()
    assert sha(pool) == str(z["sha_pool_final"])


@pytest.mark.parametrize("name", ENGINE_GOLDEN_NAMES)
def test_oracle_pre_attention_matches_engine(name, oracle):
    """q/k RMSNorm + rotary of the raw projections, with the rotary table the
    engine applies (its model.to(dtype), engine.py:84, keeps only the real part
    of the complex freqs_cis: cos, no sin), reproduce the q and k rows the engine
    produced: within 1e-6 of the row's largest magnitude in fp32, 2^-6 in bf16
    (torch's CPU rsqrt rounds the square root before the reciprocal)."""
    z, _ = load_engine_golden(name)
    td = torch.float32 if str(z["dtype"]) == "float32" else torch.bfloat16
    tol = 1e-6 if td == torch.float32 else 2.0 ** -6
    rope = torch.from_numpy(z["rope_engine"])
    assert np.all(z["rope_engine"][..., 1] == 0)
    for s in range(int(z["steps"])):
        pos = z["total"][s] - 1
        for l in range(int(z["num_layers"])):
            t = lambda a: torch.from_numpy(a).to(td)  # noqa: E731
            q, k, _ = oracle.qk_norm_rope(t(z["q_raw"][s, l]), t(z["k_raw"][s, l]), t(z["q_norm_w"][l]),
                                          t(z["k_norm_w"][l]), rope, pos, float(z["eps"]))
            for got, want in ((q, z["q"][s, l]), (k, z["k_rows"][s, l])):
                rel = np.abs(np.asarray(got, np.float32) - want).max(-1) / np.abs(want).max(-1)
                assert rel.max() <= tol, rel.max()
