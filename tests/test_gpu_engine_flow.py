"""GPU: the reference engine's decode flow driven through this package's drop-ins.

Replays the fixtures of tests/golden/make_engine_golden.py -- three decode
steps of the reference ``InferenceEngine.decode_step`` (engine.py:157-234) over
a small random model (head_dim 112, GQA 2, 3 layers), fp32 and bf16 -- on
cuda:0, starting from the pool prefill left. Per step the block table and
lengths are built as at engine.py:179-185; per layer the engine's K/V rows are
appended at total_len - 1 (:213-215) and attention runs over total_len
positions (:221-224) through:

* ``separate``: ``slot_mapping`` + ``kv_append`` + the drop-in
  ``paged_decode_attention(q, k_pool, v_pool, block_tables, seq_lens,
  block_size)``, the call the engine makes;
* ``fused``: ``paged_decode_append_attention``, append and attention in one launch;
* ``prep``: from the raw q/k projections, q/k RMSNorm + rotary + append +
  attention (``paged_decode_prep_attention``; fp32 as two launches); the rotated
  q must match the q the engine handed to attention (within 1e-6 of the row's
  largest magnitude in fp32, 2^-6 in bf16, where torch's CPU rsqrt rounds
  twice). The rotary table is the one the engine applies: its model.to(dtype)
  (engine.py:84) casts the complex freqs_cis buffer to a real one, so the engine
  multiplies by cos and drops sin, in every dtype; the kernels take that table
  as (cos, 0) pairs.

After every append the layer's pools have the engine's bytes (SHA-256); every
output meets the attention tolerance against the fp32 evaluation of the
reference (fp32 max-abs 1e-5; bf16 max-abs 2e-2, mean-abs 2e-3; the prep
variant 5e-5, its q being rotated here rather than taken from the engine) and,
for bf16, against the engine's own bf16 output too.
"""
import numpy as np
import pytest
import torch

from conftest import ENGINE_GOLDEN_NAMES, engine_block_table, load_engine_golden, sha

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

VARIANTS = [(n, v) for n in ENGINE_GOLDEN_NAMES for v in ("separate", "fused", "prep")]


def _err(out, ref):
    e = np.abs(out.float().cpu().numpy().astype(np.float64) - ref.astype(np.float64))
    return e.max(), e.mean()


@pytest.mark.parametrize("name,variant", VARIANTS)
def test_engine_decode_flow(name, variant, pkg):
    z, pool_h = load_engine_golden(name)
    td = pool_h.dtype
    pool = pool_h.to(DEV)
    L, S, bs = int(z["num_layers"]), int(z["steps"]), int(z["block_size"])
    tol = {"float32": (5e-5 if variant == "prep" else 1e-5, 1e-6), "bfloat16": (2e-2, 2e-3)}[str(z["dtype"])]
    rope = torch.from_numpy(z["rope_engine"]).to(DEV)
    q_tol = 1e-6 if td == torch.float32 else 2.0 ** -6
    for s in range(S):
        bt = torch.from_numpy(engine_block_table(z["blocks"][s])).to(DEV)
        seq_lens = torch.from_numpy(z["total"][s].astype(np.int32)).to(DEV)
        for l in range(L):
            k_pool, v_pool = pool[l, 0], pool[l, 1]          # KVPool.get_kv_layer (kvcache.py:264-266)
            k_rows = torch.from_numpy(z["k_rows"][s, l]).to(td).to(DEV)
            v_rows = torch.from_numpy(z["v_rows"][s, l]).to(td).to(DEV)
            q = torch.from_numpy(z["q"][s, l]).to(td).to(DEV)
            if variant == "separate":
                slots = pkg.slot_mapping(bt, seq_lens - 1, bs)
                pkg.kv_append(k_rows, v_rows, k_pool, v_pool, slots)
                out = pkg.paged_decode_attention(q, k_pool, v_pool, bt, seq_lens, bs)
            elif variant == "fused":
                out = pkg.paged_decode_append_attention(q, k_rows, v_rows, k_pool, v_pool, bt, seq_lens)
            else:
                q_raw = torch.from_numpy(z["q_raw"][s, l]).to(td).to(DEV)
                k_raw = torch.from_numpy(z["k_raw"][s, l]).to(td).to(DEV)
                qw = torch.from_numpy(z["q_norm_w"][l]).to(td).to(DEV)
                kw = torch.from_numpy(z["k_norm_w"][l]).to(td).to(DEV)
                q_rot, _ = pkg.qk_norm_rope(q_raw, k_raw, qw, kw, rope, seq_lens - 1, float(z["eps"]),
                                            return_k=False)
                dq = (q_rot.float() - q.float()).abs().amax(dim=-1) / q.float().abs().amax(dim=-1)
                assert dq.max().item() <= q_tol, dq.max().item()
                out = pkg.paged_decode_prep_attention(q_raw, k_raw, v_rows, qw, kw, rope, k_pool, v_pool, bt,
                                                      seq_lens, float(z["eps"]))
            torch.cuda.synchronize()
            pkg.check_device_errors()
            if variant != "prep":
                assert sha(k_pool.cpu()) == str(z["sha_k_after"][s, l]), (s, l)
                assert sha(v_pool.cpu()) == str(z["sha_v_after"][s, l]), (s, l)
            else:
                # the rotated k row is this package's; the V rows and every other slot are the engine's
                assert sha(v_pool.cpu()) == str(z["sha_v_after"][s, l]), (s, l)
            assert out.dtype == td and out.shape == q.shape
            mx, mean = _err(out, z["out_ref32"][s, l])
            assert mx <= tol[0] and mean <= tol[1], (s, l, mx, mean)
            if td == torch.bfloat16:
                mx, mean = _err(out, z["out_engine"][s, l])
                assert mx <= 2e-2 and mean <= 2e-3, (s, l, mx, mean)
    if variant != "prep":
        assert sha(pool.cpu()) == str(z["sha_pool_final"])
