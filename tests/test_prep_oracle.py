"""CPU: the pre-attention oracle (q/k RMSNorm + rotary embedding, oracle/oracle.py)
is pinned to the reference's own outputs (golden fixtures made by running
unbox_platform/model/model.py's RMSNorm, apply_rotary_emb and
precompute_freqs_cis, and PagedKVCache.write_kv, the way the engine calls them).

Tolerance. The oracle rounds where torch's CUDA kernels round (each op's fp32
result once to the dtype). torch's CPU rsqrt for bf16/f16 rounds the square
root to the dtype before taking the reciprocal, so on the CPU-made fixtures the
norm factor of some rows is 1-2 units in the last place away from the
single-rounded one. Every element must lie within 2**-6 (bf16), 2**-9 (f16) or
1e-6 (fp32) of the largest magnitude in its head row.
"""
import numpy as np
import pytest
import torch

from conftest import PREP_GOLDEN_NAMES, load_prep_golden, sha

ROW_TOL = {"bfloat16": 2.0 ** -6, "float16": 2.0 ** -9, "float32": 1e-6}


def row_close(a: np.ndarray, ref: np.ndarray, dtype: str):
    scale = np.abs(ref).max(axis=-1, keepdims=True)
    err = np.abs(a - ref) / np.maximum(scale, 1e-30)
    return float(err.max()), float((a != ref).mean())


@pytest.mark.parametrize("name", PREP_GOLDEN_NAMES)
def test_prep_oracle_matches_reference_golden(name, oracle):
    z, lay, x, caches, rope = load_prep_golden(name)
    dtype = str(z["dtype"])
    q, k, bad = oracle.qk_norm_rope(x["q_raw"], x["k_raw"], x["q_weight"], x["k_weight"], rope, z["positions"],
                                    float(z["eps"]))
    assert not bad.any()
    for what, a, ref in (("q", q, z["q_rot_ref"]), ("k", k, z["k_rot_ref"])):
        rel, neq = row_close(a, ref, dtype)
        assert rel <= ROW_TOL[dtype], (what, rel, neq)


@pytest.mark.parametrize("name", PREP_GOLDEN_NAMES)
def test_prep_oracle_append_matches_reference_pool(name, oracle):
    """The write: V rows and every untouched slot are bit-identical to the
    reference pool; the K rows written are the oracle's rotated k."""
    z, lay, x, caches, rope = load_prep_golden(name)
    dtype = str(z["dtype"])
    td = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[dtype]
    _, k, _ = oracle.qk_norm_rope(x["q_raw"], x["k_raw"], x["q_weight"], x["k_weight"], rope, z["positions"],
                                  float(z["eps"]))
    if str(z["kind"]) == "decode":
        slots = z["slot_mapping"]
    else:
        row = z["block_table_row"][None, :].repeat(int(z["num_tokens"]), 0)
        slots, st = oracle.slot_mapping(row, z["positions"], int(z["block_size"]))
        assert st == 0
    kc, vc = caches["k_cache"].clone(), caches["v_cache"].clone()
    assert oracle.kv_append(torch.from_numpy(k).to(td), x["v_new"], kc, vc, torch.from_numpy(slots)) == 0
    assert sha(vc) == str(z["sha_v_after"])
    if sha(kc) == str(z["sha_k_after"]):
        return  # every rotated k row equals the reference's
    # only the written K rows may differ, and only within the rounding tolerance
    NB, bs = kc.shape[0], kc.shape[1]
    written = np.zeros(NB * bs, dtype=bool)
    written[slots[slots >= 0]] = True
    kc_rows = kc.float().numpy().reshape(NB * bs, -1)
    base_rows = caches["k_cache"].float().numpy().reshape(NB * bs, -1)
    assert np.array_equal(kc_rows[~written], base_rows[~written])
    ref = z["k_rot_ref"].reshape(len(slots), -1)
    rel, _ = row_close(kc_rows[slots], ref, dtype)
    assert rel <= ROW_TOL[dtype]


def test_rope_table_is_the_reference_table(pkg):
    """ops.rope_table (our restatement of precompute_freqs_cis) reproduces the
    reference's table rows stored in the fixtures, bit for bit."""
    from unbox_b200 import ops
    for name in PREP_GOLDEN_NAMES:
        z, *_ = load_prep_golden(name)
        tab = ops.rope_table(int(z["head_dim"]), int(z["rope_positions"]), float(z["theta"]))
        assert np.array_equal(tab.numpy()[z["positions"]], z["rope_rows"]), name


def test_rounding_helpers(oracle):
    # bf16 round-to-nearest-even, ties to even
    a = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 1e-40], dtype=np.float32)
    r = oracle.round_to(a, oracle.BF16)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == 1.0 + 2 ** -6 and r[3] == -2.5
    assert np.array_equal(oracle.round_to(a, oracle.F32), a)
    # RMSNorm fp32 path against the float64 formula
    x = np.random.default_rng(0).standard_normal((4, 112)).astype(np.float32)
    w = np.ones(112, dtype=np.float32)
    y = oracle.rms_norm(x, w, 1e-6, oracle.F32)
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-6)
    assert np.abs(y - ref).max() < 1e-5


def test_bad_position_is_reported_and_unrotated(oracle):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 2, 8, generator=g)
    k = torch.randn(2, 1, 8, generator=g)
    w = torch.ones(8)
    rope = torch.zeros(4, 4, 2)
    rope[..., 0] = 1.0
    q, kk, bad = oracle.qk_norm_rope(x, k, w, w, rope, np.array([1, 9]), 1e-6)
    assert bad.tolist() == [False, True]
    np.testing.assert_allclose(q[1], oracle.rms_norm(x[1].numpy(), w.numpy(), 1e-6, oracle.F32))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_sixteen_bit_products_are_exact_in_fp32(dtype):
    """The kernels' norm multiplies two 16-bit values with one packed 16-bit
    multiply instead of an fp32 multiply followed by a rounding to the dtype.
    Both give the same value because the exact product of two bf16 (or two
    fp16) values fits an fp32 significand whenever it is a normal fp32 number:
    checked here against float64 on values spread over the whole range, with
    the one-rounding result (float64 product rounded once to the dtype) equal to
    the two-rounding one (fp32 product rounded to the dtype)."""
    g = torch.Generator().manual_seed(7)
    n = 200_000
    finfo = torch.finfo(dtype)
    mag = torch.exp2(torch.empty(n).uniform_(-40.0, 40.0, generator=g)) if dtype == torch.bfloat16 else \
        torch.exp2(torch.empty(n).uniform_(-12.0, 12.0, generator=g))
    sign = torch.where(torch.rand(n, generator=g) < 0.5, -1.0, 1.0)
    a = (mag * sign).to(dtype)
    b = (torch.exp2(torch.empty(n).uniform_(-20.0, 20.0, generator=g)) * sign.flip(0)).to(dtype)
    if dtype == torch.float16:
        b = (torch.exp2(torch.empty(n).uniform_(-6.0, 6.0, generator=g)) * sign.flip(0)).to(dtype)
    exact = a.double() * b.double()
    f32 = a.float() * b.float()
    normal = (exact.abs() >= torch.finfo(torch.float32).tiny) & (exact.abs() <= torch.finfo(torch.float32).max)
    assert normal.float().mean() > 0.99
    assert torch.equal(f32.double()[normal], exact[normal])                      # no rounding in fp32
    in_range = normal & (exact.abs() <= finfo.max)
    assert torch.equal(f32[in_range].to(dtype), exact[in_range].to(dtype))       # one rounding = two
