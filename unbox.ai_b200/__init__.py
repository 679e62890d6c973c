"""unbox_b200: B200-native paged decode attention and KV append for the unbox.ai engine.

The package directory is ``unbox.ai_b200/`` and it is imported under the name
``unbox_b200`` (the directory name is not a Python identifier), e.g.::

    import importlib.util, sys
    spec = importlib.util.spec_from_file_location(
        "unbox_b200", "<repo>/unbox.ai_b200/__init__.py",
        submodule_search_locations=["<repo>/unbox.ai_b200"])
    unbox_b200 = importlib.util.module_from_spec(spec)
    sys.modules["unbox_b200"] = unbox_b200
    spec.loader.exec_module(unbox_b200)

Public API (mirrors unbox_platform/infer/kernels/paged_decode_attention.py and
unbox_platform/infer/kvcache.py of the reference):

* ``paged_decode_attention(q, k_pool, v_pool, block_tables, seq_lens, block_size)``
  -- drop-in for the reference function of the same name (engine.py:221-224).
* ``paged_attention(q, k_cache, v_cache, block_table, context_lens, scale)``
  -- the same op with an explicit softmax scale.
* ``kv_append(k_new, v_new, k_cache, v_cache, slot_mapping)`` -- batched
  replacement for the per-sequence ``PagedKVCache.write_kv`` loop.
* ``paged_decode_append_attention(q, k_new, v_new, k_cache, v_cache, block_table,
  context_lens, scale)`` -- the append and the attention of one decode layer
  in a single launch.
* ``slot_mapping(block_table, positions, block_size)`` -- device-side slot
  computation (kvcache.py:338-339) for one decode step.
* ``qk_norm_rope(q, k, q_weight, k_weight, rope, positions, eps, ...)`` -- the
  q/k RMSNorm and rotary embedding of T tokens (model.py:19-48 as used at
  engine.py:201-210), optionally with the KV append, in one launch.
* ``paged_decode_prep_attention(q_raw, k_raw, v_new, q_weight, k_weight, rope,
  k_cache, v_cache, block_table, context_lens, eps)`` -- norm, rotary, append
  and attention of one decode layer (engine.py:201-224) in one launch.
* ``prefill_kv_write`` / ``prefill_prep`` -- a prefill chunk's KV write
  (engine.py:126-128), alone or with its norm and rotary steps (:121-128);
  ``prefill_positions_and_slots`` computes the chunk's positions and slots once
  per step for all layers.
* ``rope_table(head_dim, num_positions, theta)`` -- the (cos, sin) table of
  precompute_freqs_cis (model.py:30-34).
* ``plan_cascade(block_table, context_lens, H, KVH)`` /
  ``paged_attention_cascade(q, k_cache, v_cache, plan, ...)`` -- decode attention
  that reads radix-shared prefix pages once per step for all requests sharing
  them (kvcache.py:97-122 produces such tables).
* ``handoff`` -- KV page hand-off between workers: ``serialize_blocks`` /
  ``deserialize_blocks`` (kvcache.py:268-277) on the device with a typed
  header, and ``transfer_pages`` pool to pool over NVLink.
"""
from . import workloads  # noqa: F401  (pure Python, no CUDA needed)

__all__ = [
    "paged_decode_attention", "paged_attention", "paged_attention_split", "kv_append",
    "slot_mapping", "DecodeWorkspace", "workloads", "library", "sharding", "qk_norm_rope",
    "paged_decode_prep_attention", "prefill_kv_write", "prefill_prep", "prefill_slots",
    "prefill_positions_and_slots", "rope_table", "handoff", "cascade", "plan_cascade", "paged_attention_cascade",
]


_OPS = ("paged_decode_attention", "paged_attention", "paged_attention_split", "kv_append", "slot_mapping",
        "DecodeWorkspace", "check_device_errors", "workspace_for", "paged_decode_append_attention",
        "qk_norm_rope", "paged_decode_prep_attention", "prefill_kv_write", "prefill_prep", "prefill_slots",
        "prefill_positions_and_slots", "rope_table")


def __getattr__(name):
    # submodules that need torch / the CUDA library load lazily, so that the
    # fixture generator and CPU-only host logic import without them
    import importlib
    if name in _OPS:
        return getattr(importlib.import_module(__name__ + ".ops"), name)
    if name in ("plan_cascade", "paged_attention_cascade", "CascadePlan"):
        return getattr(importlib.import_module(__name__ + ".cascade"), name)
    if name in ("library", "sharding", "ops", "build", "handoff", "cascade"):
        return importlib.import_module(__name__ + "." + name)
    raise AttributeError(name)
