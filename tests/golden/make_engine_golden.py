"""Generate the engine-flow golden fixtures by running the reference engine's
own decode step.

Run in a container that has the reference checked out (read-only is fine):

    UNBOX_REFERENCE=<reference checkout> python tests/golden/make_engine_golden.py

(or ``--reference <checkout>``). For each case it builds the reference's
``InferenceEngine`` (unbox_platform/infer/engine.py) on the CPU around a small
randomly initialised ``UnboxForCausalLM`` (head_dim 112, GQA 2: 4 query heads,
2 KV heads, 3 layers; the checkpoint loader is the only part replaced), admits
three requests whose prompts end before, on and past a page boundary,
prefills them with ``prefill_step`` and then runs ``decode_step`` three
times, feeding back the argmax token as the scheduler would
(scheduler.py:106-110,122-124: append the token, ``ensure_blocks``, decode).
The engine is unmodified; recording wrappers sit around
``PagedKVCache.write_kv`` and the paged-attention function it calls, and
forward pre-hooks on ``q_norm`` / ``k_norm`` keep their inputs. Stored per
decode step: the sequences' block lists and total lengths (engine.py:179-185);
per step and layer: the K/V rows the engine appends at ``total_len - 1``
(:213-215), the query it hands to attention (:221-224), the attention output
(the engine's own, in the engine's dtype, and an fp32 evaluation of the same
reference function on the upcast values), the SHA-256 of the layer's pools
after the append, and for the pre-attention steps the raw q/k projections, the
norm weights and the rotary rows (as the model defines them, and as the engine
applies them after its dtype cast, which keeps only their real part). Also the
KV pool as prefill left it, from which the GPU test replays the flow.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = {
    # name: (dtype, seed)
    "engine_decode_fp32": ("float32", 0),
    "engine_decode_bf16": ("bfloat16", 1),
}
PROMPTS = (5, 16, 33)        # tokens: inside page 0, exactly one page, past two pages
STEPS, LAYERS, NUM_BLOCKS = 3, 3, 12


def sha(t) -> str:
    import torch
    x = t.detach().contiguous()
    if x.dtype == torch.bfloat16:
        x = x.view(torch.int16)
    return hashlib.sha256(x.numpy().tobytes()).hexdigest()


def f32(t):
    return t.detach().float().numpy().copy()


def run_case(ref_root, dtype, seed):
    import torch
    sys.path.insert(0, ref_root)
    from unbox_platform.infer.config import InferConfig
    from unbox_platform.infer.engine import InferenceEngine
    from unbox_platform.infer.kernels.paged_decode_attention import paged_decode_attention_ref
    from unbox_platform.infer.kvcache import SequenceState
    from unbox_platform.model.config import ModelConfig
    from unbox_platform.model.hf_adapter import UnboxConfig, UnboxForCausalLM

    mcfg = ModelConfig(hidden_size=448, num_layers=LAYERS, num_heads=4, num_kv_heads=2, ffn_intermediate_size=512,
                       vocab_size=101, max_seq_len=128)
    torch.manual_seed(seed)
    model = UnboxForCausalLM(UnboxConfig.from_model_config(mcfg))
    model._recompute_rope_buffers()
    freqs = model.model.freqs_cis.clone()          # complex64, before any dtype cast
    td = {"float32": torch.float32, "bfloat16": torch.bfloat16}[dtype]

    class Engine(InferenceEngine):
        def _load_model(self):                     # the only replaced step: no checkpoint file
            return model.to(td).eval()

    eng = Engine(InferConfig(block_size=16, max_num_blocks=NUM_BLOCKS, dtype=dtype), torch.device("cpu"))
    assert eng._paged_attn is paged_decode_attention_ref
    m = eng.model.model
    g = torch.Generator().manual_seed(100 + seed)
    seqs = []
    for i, n in enumerate(PROMPTS):
        s = SequenceState(request_id=f"r{i}", prompt_token_ids=torch.randint(0, 101, (n,), generator=g).tolist())
        eng.kvcache.prepare_sequence(s)
        eng.kvcache.ensure_blocks(s)
        logits = eng.prefill_step(s, s.prompt_token_ids, 0)
        s.prefill_cursor = n
        s.generated_token_ids.append(int(logits.float().argmax()))
        seqs.append(s)
    pool0 = eng.kvcache._pool.data.clone()

    rec = {"write": [], "attn": [], "qn": [], "kn": []}
    orig_write = eng.kvcache.write_kv

    def write_kv(layer_idx, seq, token_pos, k, v):
        rec["write"].append((layer_idx, seqs.index(seq), token_pos, k.clone(), v.clone()))
        return orig_write(layer_idx, seq, token_pos, k, v)

    def attn(q, k_pool, v_pool, block_tables, seq_lens, block_size):
        out = paged_decode_attention_ref(q, k_pool, v_pool, block_tables, seq_lens, block_size)
        out32 = paged_decode_attention_ref(q.float(), k_pool.float(), v_pool.float(), block_tables, seq_lens,
                                           block_size)
        rec["attn"].append(dict(q=q.clone(), bt=block_tables.clone(), sl=seq_lens.clone(), out=out.clone(),
                                out32=out32, sha_k=sha(k_pool), sha_v=sha(v_pool)))
        return out

    eng.kvcache.write_kv = write_kv
    eng._paged_attn = attn
    hooks = []
    for layer in m.layers:
        hooks.append(layer.attn.q_norm.register_forward_pre_hook(lambda mod, a: rec["qn"].append(a[0].clone())))
        hooks.append(layer.attn.k_norm.register_forward_pre_hook(lambda mod, a: rec["kn"].append(a[0].clone())))

    steps = []
    for step in range(STEPS):
        for s in seqs:
            eng.kvcache.ensure_blocks(s)          # scheduler.py:110, before the decode step
        blocks = [list(s.block_table) for s in seqs]
        total = [s.total_len for s in seqs]
        tokens = [s.generated_token_ids[-1] for s in seqs]
        for k in rec:
            rec[k].clear()
        logits = eng.decode_step(seqs, tokens)
        assert len(rec["attn"]) == LAYERS and len(rec["write"]) == LAYERS * len(seqs)
        steps.append(dict(blocks=blocks, total=total, attn=list(rec["attn"]), write=list(rec["write"]),
                          qn=list(rec["qn"]), kn=list(rec["kn"])))
        for i, s in enumerate(seqs):
            s.generated_token_ids.append(int(logits[i].float().argmax()))
    for h in hooks:
        h.remove()

    B, H, KVH, D = len(seqs), mcfg.num_heads, mcfg.num_kv_heads, mcfg.head_dim
    maxblk = max(len(b) for st in steps for b in st["blocks"])
    out = dict(dtype=np.array(dtype), seed=np.array(seed), num_layers=np.array(LAYERS), num_heads=np.array(H),
               num_kv_heads=np.array(KVH), head_dim=np.array(D), block_size=np.array(16),
               num_blocks=np.array(NUM_BLOCKS), steps=np.array(STEPS), eps=np.array(mcfg.rms_norm_eps),
               pool0=f32(pool0), sha_pool0=np.array(sha(pool0)))
    blocks = np.full((STEPS, B, maxblk), -1, dtype=np.int32)
    total = np.zeros((STEPS, B), dtype=np.int32)
    q = np.zeros((STEPS, LAYERS, B, H, D), np.float32)
    q_raw = np.zeros_like(q)
    k_raw = np.zeros((STEPS, LAYERS, B, KVH, D), np.float32)
    k_rows, v_rows = np.zeros_like(k_raw), np.zeros_like(k_raw)
    out_eng, out32 = np.zeros_like(q), np.zeros_like(q)
    bt_rec = np.full((STEPS, B, maxblk), -2, dtype=np.int32)
    sl_rec = np.zeros((STEPS, B), dtype=np.int32)
    sha_k = np.zeros((STEPS, LAYERS), dtype="U64")
    sha_v = np.zeros_like(sha_k)
    for si, st in enumerate(steps):
        for b, bl in enumerate(st["blocks"]):
            blocks[si, b, :len(bl)] = bl
        total[si] = st["total"]
        for l, a in enumerate(st["attn"]):
            q[si, l], out_eng[si, l], out32[si, l] = f32(a["q"]), f32(a["out"]), f32(a["out32"])
            bt_rec[si, :, :a["bt"].shape[1]] = a["bt"].numpy()
            sl_rec[si] = a["sl"].numpy()
            sha_k[si, l], sha_v[si, l] = a["sha_k"], a["sha_v"]
            q_raw[si, l] = f32(st["qn"][l][:, 0])
            k_raw[si, l] = f32(st["kn"][l][:, 0])
        for (l, b, pos, k, v) in st["write"]:
            assert pos == st["total"][b] - 1
            k_rows[si, l, b], v_rows[si, l, b] = f32(k), f32(v)
    # rotary rows of the decode positions, fp32 (cos, sin): as the model defines
    # them (precompute_freqs_cis), and as the engine applies them -- its
    # model.to(dtype) (engine.py:84) casts the complex freqs_cis buffer to a real
    # tensor, keeping cos and dropping sin, for every dtype
    pos = np.unique(total - 1)
    rope = np.zeros((int(pos.max()) + 1, D // 2, 2), np.float32)
    rope[pos] = torch.view_as_real(freqs[torch.from_numpy(pos)]).numpy()
    applied = m.freqs_cis
    assert not applied.is_complex(), "the engine's cast keeps only the real part of freqs_cis"
    rope_engine = np.zeros_like(rope)
    rope_engine[pos, :, 0] = applied[torch.from_numpy(pos)].float().numpy()
    qw = np.stack([f32(layer.attn.q_norm.weight) for layer in m.layers])
    kw = np.stack([f32(layer.attn.k_norm.weight) for layer in m.layers])
    out.update(blocks=blocks, total=total, block_table_rec=bt_rec, seq_lens_rec=sl_rec, q=q, q_raw=q_raw,
               k_raw=k_raw, k_rows=k_rows, v_rows=v_rows, out_engine=out_eng, out_ref32=out32, sha_k_after=sha_k,
               sha_v_after=sha_v, rope=rope, rope_engine=rope_engine, q_norm_w=qw, k_norm_w=kw, sha_pool_final=np.array(
                   sha(eng.kvcache._pool.data)))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("UNBOX_REFERENCE"),
                    help="reference checkout (default: $UNBOX_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or UNBOX_REFERENCE")
    for name, (dtype, seed) in CASES.items():
        rec = run_case(args.reference, dtype, seed)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **rec)
        print(f"{name}: {int(rec['steps'])} decode steps x {int(rec['num_layers'])} layers -> {os.path.basename(path)}")


if __name__ == "__main__":
    main()
