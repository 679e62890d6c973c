/*
 * unbox_b200 -- C ABI of the B200 (sm_100a) paged decode-attention path.
 *
 * These entry points replace, for one decode step of the unbox.ai inference
 * engine, the per-sequence KV write loop and the paged attention call
 * (reference: unbox_platform/infer/engine.py:213-224). All pointers are device
 * pointers unless stated otherwise; strides are in ELEMENTS; the innermost
 * (head_dim) dimension of every tensor is contiguous. Every call is
 * asynchronous on `stream` (a cudaStream_t passed as void*, NULL = legacy
 * default stream), allocates nothing, and never synchronises the host (except
 * ubx_read_device_error); a decode step made of ubx_slot_mapping, ubx_kv_append,
 * ubx_paged_decode_attention and ubx_paged_decode_append_attention calls can be
 * captured in a CUDA graph.
 *
 * Return value: UBX_OK or a UBX_ERR_* status for host-side validation and
 * launch failures (ubx_last_error() gives the message). Data-dependent problems
 * found on the device (a page id outside the pool, a context longer than its
 * block-table row, ...) do not fault: the kernel skips the access, writes a
 * UBX_DEVERR_* bit into the workspace's error word and carries on; read it with
 * ubx_read_device_error().
 */
#ifndef UNBOX_B200_H_
#define UNBOX_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types of q / k / v / out (the pool dtype, configs/infer/serve.yaml `dtype`) */
#define UBX_DTYPE_F32 0
#define UBX_DTYPE_BF16 1
#define UBX_DTYPE_F16 2

/* host-side status codes */
#define UBX_OK 0
#define UBX_ERR_INVALID_ARGUMENT 1 /* shape, stride, alignment or pointer rejected */
#define UBX_ERR_UNSUPPORTED 2      /* valid but not built: head_dim, block_size, GQA ratio */
#define UBX_ERR_WORKSPACE 3        /* workspace missing or too small */
#define UBX_ERR_CUDA 4             /* a CUDA runtime/driver call failed */

/* device error bits, OR-ed into the workspace error word */
#define UBX_DEVERR_BAD_PAGE 1      /* block-table entry outside [0, num_blocks): tile read as zeros */
#define UBX_DEVERR_CTX_TOO_LONG 2  /* context_len > max_blocks_per_seq * block_size: clamped */
#define UBX_DEVERR_NEG_CTX 4       /* negative context_len: treated as 0 */
#define UBX_DEVERR_TIMEOUT 8       /* a pipeline wait exceeded its bound; output undefined */
#define UBX_DEVERR_BAD_SLOT 16     /* kv_append slot >= num_blocks * block_size: row skipped */
#define UBX_DEVERR_BAD_POSITION 32 /* rotary position outside [0, rope_positions): row left unrotated */
#define UBX_DEVERR_BAD_WORK 64     /* cascade work or merge item out of range: item skipped */

/* work schedules of the attention kernel */
#define UBX_SCHEDULE_AUTO 0     /* library picks */
#define UBX_SCHEDULE_BALANCED 1 /* persistent grid, equal pages per CTA, in-kernel LSE merge */
#define UBX_SCHEDULE_SPLIT 2    /* fixed split-KV chunks per sequence + LSE combine kernel */

/* call flags (ubx_paged_decode_append_attention) */
#define UBX_FLAG_OVERLAP_PREVIOUS 1 /* launch with programmatic dependent launch: the kernel may start, and
                                       stream pool pages, while the previous kernel on the stream is still
                                       running. The caller promises that kernel writes neither the K/V pool,
                                       block_table nor context_lens (true in a decode step, where it is the
                                       previous layer's attention or this layer's QKV projection). q, k_new,
                                       v_new, out and the workspace are only touched after it completed. */

const char* ubx_status_string(int status);
/* Message of the last failing call on this host thread ("" if none). */
const char* ubx_last_error(void);
/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int ubx_version(void);

/*
 * KV append: k_cache[slot / bs, slot % bs, h, :] = k_new[t, h, :] (and V) for
 * every token t with slot = slot_mapping[t] >= 0; a negative slot is padding.
 * Byte copy, bit-exact.
 * Replaces: KVPool.write_kv (unbox_platform/infer/kvcache.py:253-262) reached
 * through PagedKVCache.write_kv (kvcache.py:330-340) once per sequence from
 * InferenceEngine.decode_step (unbox_platform/infer/engine.py:213-215).
 *   k_new, v_new:  (num_tokens, num_kv_heads, head_dim), strides (new_s_tok, new_s_head)
 *   k_cache, v_cache: (num_blocks, block_size, num_kv_heads, head_dim) -- the
 *                  per-layer views KVPool.get_kv_layer returns (kvcache.py:264-266),
 *                  strides (c_s_block, c_s_tok, c_s_head), identical for K and V
 *   slot_mapping:  (num_tokens,) int64
 *   error_word:    device int32 for UBX_DEVERR_BAD_SLOT, may be NULL
 */
int ubx_kv_append(const void* k_new, const void* v_new, int64_t new_s_tok, int64_t new_s_head,
                  void* k_cache, void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                  const int64_t* slot_mapping, int64_t num_tokens, int num_kv_heads, int head_dim,
                  int block_size, int64_t num_blocks, int dtype, int32_t* error_word, void* stream);

/*
 * Prefill chunk KV write: the K/V rows of tokens t = 0 .. num_tokens-1 of one
 * sequence, at positions start_pos + t, go to slot = block_table_row[pos // bs]
 * * bs + pos % bs (no slot, nothing written, for a position past the row's
 * max_blocks_per_seq entries or a negative page, as in ubx_slot_mapping; a page
 * outside the pool sets UBX_DEVERR_BAD_SLOT). One launch, slots computed in the
 * kernel; slots_out (num_tokens,) int64 receives them when not NULL.
 * Replaces: the per-token PagedKVCache.write_kv loop of prefill_step
 * (unbox_platform/infer/engine.py:126-128, kvcache.py:330-340).
 * Strides as in ubx_kv_append (k, v share s_tok / s_head). flags:
 * UBX_FLAG_OVERLAP_PREVIOUS = programmatic dependent launch (the kernel may
 * start while the previous kernel on the stream drains; it reads and writes
 * nothing before that kernel has completed).
 */
int ubx_prefill_kv_write(const void* k, const void* v, int64_t s_tok, int64_t s_head, void* k_cache, void* v_cache,
                         int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head, const int32_t* block_table_row,
                         int max_blocks_per_seq, int64_t start_pos, int64_t num_tokens, int num_kv_heads, int head_dim,
                         int block_size, int64_t num_blocks, int dtype, int64_t* slots_out, int32_t* error_word,
                         int flags, void* stream);

/*
 * Slot mapping of one decode step: slot[b] = block_table[b, pos // bs] * bs + pos % bs
 * with pos = positions[b] (the index arithmetic of PagedKVCache.write_kv,
 * kvcache.py:338-339). A negative position or page gives slot -1.
 * Computed once per step and shared by all layers (engine.py:179-187 builds the
 * block table once per step).
 */
int ubx_slot_mapping(const int32_t* block_table, int64_t bt_s_row, const int32_t* positions,
                     int64_t* slot_mapping, int batch, int max_blocks_per_seq, int block_size, void* stream);

/*
 * Bytes of device workspace the attention entry points need for these sizes on
 * the current device (partial results of split sequences, merge counters, the
 * error word; sized for up to 4 CTAs per SM). The workspace must be 16-byte
 * aligned and zeroed once with ubx_workspace_init before its first use; the
 * kernels leave it ready for the next call.
 */
int ubx_paged_decode_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim, int max_blocks_per_seq,
                                    int split_pages, int dtype, size_t* bytes);
int ubx_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/*
 * Paged GQA decode attention for one new token per sequence:
 *   out[b, h, :] = softmax_j(scale * q[b,h,:] . K_j) V_j over the first
 *   context_lens[b] positions of sequence b, position j living in page
 *   block_table[b, j // block_size], slot j % block_size, KV head
 *   h // (num_heads / num_kv_heads).
 * Replaces: paged_decode_attention / paged_decode_attention_ref
 * (unbox_platform/infer/kernels/paged_decode_attention.py:106-150, 157-191),
 * called at unbox_platform/infer/engine.py:221-224 with
 * scale = head_dim ** -0.5 (paged_decode_attention.py:134,169).
 *   q:            (batch, num_heads, head_dim), strides (q_s_b, q_s_h)
 *   k/v_cache:    (num_blocks, block_size, num_kv_heads, head_dim), strides
 *                 (c_s_block, c_s_tok, c_s_head) with c_s_head == head_dim
 *                 (heads of a token row contiguous, the KVPool layout); base
 *                 16-byte aligned, strides multiples of 16 bytes
 *   block_table:  (batch, max_blocks_per_seq) int32, row stride bt_s_row, -1 padded
 *   context_lens: (batch,) int32, includes the token just appended
 *   out:          (batch, num_heads, head_dim), strides (o_s_b, o_s_h), dtype of q
 * A sequence with context_len 0 gets a zero row (the reference raises there).
 * Supported: head_dim 64/112/128, block_size 16, num_heads/num_kv_heads in {1,2,4,8},
 * dtype f32/bf16/f16 (q, caches and out share it).
 */
int ubx_paged_decode_attention(const void* q, int64_t q_s_b, int64_t q_s_h, const void* k_cache,
                               const void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                               const int32_t* block_table, int64_t bt_s_row, const int32_t* context_lens,
                               void* out, int64_t o_s_b, int64_t o_s_h, int batch, int num_heads,
                               int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                               int max_blocks_per_seq, float scale, int dtype, int schedule, int split_pages,
                               void* workspace, size_t workspace_bytes, void* stream);

/*
 * KV append fused into paged decode attention: for every sequence b with
 * context_lens[b] >= 1 the rows k_new[b], v_new[b] are first written to
 * position context_lens[b] - 1 (page block_table[b, pos // bs], slot pos % bs),
 * then out is computed over all context_lens[b] positions, as
 * ubx_kv_append with slot_mapping = that slot followed by
 * ubx_paged_decode_attention would do, in one launch.
 * Replaces: the append loop and attention call of one layer of
 * InferenceEngine.decode_step (unbox_platform/infer/engine.py:213-224), with
 * the slot arithmetic of PagedKVCache.write_kv (kvcache.py:338-339).
 *   k_new, v_new: (batch, num_kv_heads, head_dim), strides (new_s_tok, new_s_head)
 *   flags:        0 or UBX_FLAG_OVERLAP_PREVIOUS
 * The other arguments are those of ubx_paged_decode_attention.
 */
int ubx_paged_decode_append_attention(const void* k_new, const void* v_new, int64_t new_s_tok, int64_t new_s_head,
                                      const void* q, int64_t q_s_b, int64_t q_s_h, void* k_cache, void* v_cache,
                                      int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                                      const int32_t* block_table, int64_t bt_s_row, const int32_t* context_lens,
                                      void* out, int64_t o_s_b, int64_t o_s_h, int batch, int num_heads,
                                      int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                                      int max_blocks_per_seq, float scale, int dtype, int schedule, int split_pages,
                                      int flags, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Pre-attention step of a decode step or a prefill chunk, one launch: for every
 * token t (position positions[t]) and head, RMSNorm of the q and k head rows,
 * then the rotary embedding at that position; q_out receives the rotated q rows,
 * k_out (optional) the rotated k rows, and when k_cache is given the rotated k
 * row and the unchanged v row are stored at slot_mapping[t] (negative slot:
 * padding, not stored).
 *   RMSNorm (unbox_platform/model/model.py:25-27): y = x * rsqrt(mean(x^2) + eps) * w
 *   rotary  (model.py:36-48): (y[2j] + i y[2j+1]) * (cos + i sin) of rope row pos, pair j
 * with the rounding of the reference's tensor ops in the model dtype (every op
 * rounds its fp32 result to the dtype; fp32 tensors are not rounded).
 * Replaces: q_norm/k_norm, the per-sequence apply_rotary_emb loop and the write_kv
 * loop of InferenceEngine.decode_step (unbox_platform/infer/engine.py:201-215) and
 * of prefill_step (engine.py:121-128).
 *   q_in:  (num_tokens, num_heads, head_dim), strides (q_s_tok, q_s_head)
 *   k_in, v_in: (num_tokens, num_kv_heads, head_dim), strides (k_s_tok, k_s_head), (v_s_tok, v_s_head)
 *   q_weight, k_weight: (head_dim,) RMSNorm weights in the model dtype
 *   rope:  (rope_positions, head_dim / 2, 2) fp32 (cos, sin) pairs, row stride rope_s_pos
 *          (torch.view_as_real of the model's complex freqs_cis, model.py:30-34)
 *   positions: (num_tokens,) int32
 *   q_out: (num_tokens, num_heads, head_dim); k_out: (num_tokens, num_kv_heads, head_dim) or NULL
 *   k_cache/v_cache/slot_mapping: as ubx_kv_append, or all NULL for no append
 *   error_word: device int32 for UBX_DEVERR_BAD_POSITION / UBX_DEVERR_BAD_SLOT, may be NULL
 * head_dim even, <= 256; element pairs must be 2-element aligned (pointers and strides).
 */
int ubx_qk_norm_rope_append(const void* q_in, int64_t q_s_tok, int64_t q_s_head, const void* k_in, int64_t k_s_tok,
                            int64_t k_s_head, const void* v_in, int64_t v_s_tok, int64_t v_s_head,
                            const void* q_weight, const void* k_weight, float eps, const float* rope,
                            int64_t rope_s_pos, int rope_positions, const int32_t* positions, void* q_out,
                            int64_t qo_s_tok, int64_t qo_s_head, void* k_out, int64_t ko_s_tok, int64_t ko_s_head,
                            void* k_cache, void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                            const int64_t* slot_mapping, int64_t num_blocks, int block_size, int64_t num_tokens,
                            int num_heads, int num_kv_heads, int head_dim, int dtype, int32_t* error_word,
                            void* stream);

/*
 * One launch per layer for the whole attention block of a decode step between the
 * QKV projection and o_proj: RMSNorm + rotary embedding of q and of the new k
 * row at position context_lens[b] - 1 (as ubx_qk_norm_rope_append), the KV append
 * of that k row and of v_new, and paged decode attention over all
 * context_lens[b] positions (as ubx_paged_decode_append_attention).
 * Replaces: engine.py:201-224 of InferenceEngine.decode_step.
 *   q_raw:  (batch, num_heads, head_dim) q projection, strides (q_s_b, q_s_h)
 *   k_raw, v_new: (batch, num_kv_heads, head_dim) k and v projections, strides (new_s_tok, new_s_head)
 *   q_weight, k_weight, eps, rope, rope_s_pos, rope_positions: as ubx_qk_norm_rope_append
 * The other arguments are those of ubx_paged_decode_append_attention. Built for
 * bf16 and f16 (fp32: UBX_ERR_UNSUPPORTED, run ubx_qk_norm_rope_append and then
 * ubx_paged_decode_attention).
 */
int ubx_paged_decode_prep_attention(const void* q_raw, int64_t q_s_b, int64_t q_s_h, const void* k_raw,
                                    const void* v_new, int64_t new_s_tok, int64_t new_s_head, const void* q_weight,
                                    const void* k_weight, float eps, const float* rope, int64_t rope_s_pos,
                                    int rope_positions, void* k_cache, void* v_cache, int64_t c_s_block,
                                    int64_t c_s_tok, int64_t c_s_head, const int32_t* block_table, int64_t bt_s_row,
                                    const int32_t* context_lens, void* out, int64_t o_s_b, int64_t o_s_h, int batch,
                                    int num_heads, int num_kv_heads, int head_dim, int block_size,
                                    int64_t num_blocks, int max_blocks_per_seq, float scale, int dtype, int schedule,
                                    int split_pages, int flags, void* workspace, size_t workspace_bytes,
                                    void* stream);

/*
 * ubx_paged_decode_append_attention that also returns, per (sequence, query
 * head), lse_out[b * num_heads + h] = log2 of the softmax denominator in the
 * exp2 domain: max_j(s_j) + log2(sum_j 2^(s_j - max)), s_j = scale * log2(e) *
 * q . K_j (-inf for an empty context). k_new / v_new may both be NULL (no
 * append). bf16/f16. Used by the cascade below (the suffix pass), so it leaves
 * 4 KB of each SM's shared memory to the small CTAs of the launches that follow
 * it with programmatic overlap; no counterpart in the reference.
 */
int ubx_paged_decode_attention_lse(const void* k_new, const void* v_new, int64_t new_s_tok, int64_t new_s_head,
                                   const void* q, int64_t q_s_b, int64_t q_s_h, void* k_cache, void* v_cache,
                                   int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head, const int32_t* block_table,
                                   int64_t bt_s_row, const int32_t* context_lens, void* out, int64_t o_s_b,
                                   int64_t o_s_h, int batch, int num_heads, int num_kv_heads, int head_dim,
                                   int block_size, int64_t num_blocks, int max_blocks_per_seq, float scale, int dtype,
                                   int schedule, int split_pages, int flags, float* lse_out, void* workspace,
                                   size_t workspace_bytes, void* stream);

/*
 * Shared-prefix (cascade) decode attention for requests whose block tables start
 * with the same pages (the radix cache's shared prompt prefix, produced by the
 * prefix match of unbox_platform/infer/kvcache.py:97-122). Attention over the
 * whole context = log-sum-exp merge of attention over the shared pages and over
 * the request's own suffix, so a step runs:
 *   1. ubx_paged_decode_attention_lse over each request's suffix (its block-table
 *      row from the first unshared page, context minus the shared tokens), with
 *      the fused append, writing out and lse;
 *   2. ubx_cascade_prefix_attention: for each work item and KV head, one CTA
 *      loads up to 8 shared pages of that head once and runs all the item's
 *      (request, query head) rows over them as one 128-row tile on the tcgen05
 *      tensor cores, writing per-chunk partials into the cascade workspace;
 *   3. ubx_cascade_merge: out[b, h] = merge(suffix row with weight 2^lse, chunk partials).
 * Replaces, for those requests, the per-request re-reading of shared pages in
 * paged_decode_attention_ref (unbox_platform/infer/kernels/paged_decode_attention.py:157-191).
 *   page_list:   int32, the shared page ids of every group, concatenated
 *   member_list: int32, the member sequences of every group, concatenated
 *   work_items:  int32 [num_work_items][6] = (member offset, member count, page
 *                offset, page count <= 64 (taken 8 at a time), chunk index <
 *                max_chunks, 0); member count * (num_heads / num_kv_heads) <= 128
 *   merge_items: int32 [num_merge_items][2] = (sequence, number of its prefix chunks)
 *   cascade_ws:  ubx_cascade_workspace_size bytes, 16-byte aligned (no initialisation needed)
 *   flags:       UBX_FLAG_OVERLAP_PREVIOUS = programmatic dependent launch: the
 *                kernel may start while the previous kernel on the stream drains.
 *                The prefix pass then loads its shared pages before waiting for
 *                that kernel, and the merge reads merge_items before it (the
 *                caller promises that kernel writes neither those pages nor
 *                page_list / member_list / work_items / merge_items, which holds
 *                for the suffix pass of step 1: its append lands in private
 *                pages); q, the workspace and the outputs are touched only after
 *                the wait.
 * bf16/f16, head_dim 64/112/128, page 16, GQA 1/2/4/8.
 */
int ubx_cascade_workspace_size(int batch, int num_heads, int head_dim, int max_chunks, size_t* bytes);
int ubx_cascade_prefix_attention(const void* q, int64_t q_s_b, int64_t q_s_h, const void* k_cache,
                                 const void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                                 int64_t num_blocks, const int32_t* page_list, const int32_t* member_list,
                                 const int32_t* work_items, int num_work_items, int max_chunks, int batch,
                                 int num_heads, int num_kv_heads, int head_dim, float scale, int dtype,
                                 void* cascade_ws, size_t cascade_ws_bytes, int32_t* error_word, int flags,
                                 void* stream);
int ubx_cascade_merge(void* out, int64_t o_s_b, int64_t o_s_h, const float* lse, const int32_t* merge_items,
                      int num_merge_items, int max_chunks, int batch, int num_heads, int head_dim, int dtype,
                      const void* cascade_ws, size_t cascade_ws_bytes, int32_t* error_word, int flags,
                      void* stream);

/*
 * The whole cascade step in one call: steps 1-3 above with the arguments they
 * take (suffix_block_table / suffix_context_lens are step 1's block_table /
 * context_lens, schedule is step 1's; the device error word is the
 * workspace's). With prefix_ctas > 0, and when the suffix pass runs the
 * balanced schedule with one CTA per SM, steps 1 and 2 share one launch: its
 * first prefix_ctas CTAs (at least 1, at most the grid less one) run the work
 * items on the tensor cores while the others stream the suffix pages, on
 * disjoint SMs. Otherwise (prefix_ctas = 0, the split schedule, several CTAs
 * per SM) they are two launches. Step 3 follows.
 */
int ubx_cascade_attention(const void* k_new, const void* v_new, int64_t new_s_tok, int64_t new_s_head,
                          const void* q, int64_t q_s_b, int64_t q_s_h, void* k_cache, void* v_cache,
                          int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head, const int32_t* suffix_block_table,
                          int64_t bt_s_row, const int32_t* suffix_context_lens, void* out, int64_t o_s_b,
                          int64_t o_s_h, int batch, int num_heads, int num_kv_heads, int head_dim, int block_size,
                          int64_t num_blocks, int max_blocks_per_seq, float scale, int dtype, int schedule,
                          const int32_t* page_list, const int32_t* member_list, const int32_t* work_items,
                          int num_work_items, const int32_t* merge_items, int num_merge_items, int max_chunks,
                          int prefix_ctas, int flags, float* lse_out, void* workspace, size_t workspace_bytes,
                          void* cascade_ws, size_t cascade_ws_bytes, void* stream);

/*
 * KV hand-off between a prefill worker and a decode worker.
 * Replaces: KVPool.serialize_blocks / deserialize_blocks
 * (unbox_platform/infer/kvcache.py:268-277), used at worker.py:175-183 (prefill
 * side) and :217-223 (decode side), which copy the pages through host memory,
 * serialise only fp32 pools (bf16 raises in numpy) and decode every payload as
 * float32. Here pages move on the device, the wire message carries a fixed
 * 64-byte header with the payload's dtype and geometry, and a pool-to-pool copy
 * can write straight into another GPU's pool over NVLink.
 *
 * Wire message = ubx_kv_wire_header followed by the payload: the pages in the
 * reference's byte order, (num_layers, 2 [K, V], num_pages, block_size,
 * num_kv_heads, head_dim) in the pool dtype. All fields little-endian.
 */
#define UBX_KV_WIRE_MAGIC "UBXKVPG1"
#define UBX_KV_WIRE_VERSION 1
typedef struct ubx_kv_wire_header {
  char magic[8];          /* UBX_KV_WIRE_MAGIC, not NUL-terminated */
  uint32_t version;       /* UBX_KV_WIRE_VERSION */
  uint32_t header_bytes;  /* 64 */
  uint32_t dtype;         /* UBX_DTYPE_* of the payload */
  uint32_t num_layers;
  uint32_t num_kv_heads;
  uint32_t head_dim;
  uint32_t block_size;
  uint32_t num_pages;
  uint64_t payload_bytes; /* num_layers * 2 * num_pages * block_size * num_kv_heads * head_dim * element bytes */
  uint64_t checksum;      /* sum over the payload's 32-bit words p[i] of p[i] * (2i + 1), mod 2^64 */
  uint8_t reserved[8];    /* zero */
} ubx_kv_wire_header;

/* Fill a header (host memory). */
int ubx_kv_wire_header_init(ubx_kv_wire_header* header, int dtype, int num_layers, int num_kv_heads, int head_dim,
                            int block_size, int num_pages, uint64_t checksum);
/*
 * Check a received header (host memory) against the receiving pool's geometry
 * and the payload size that arrived: UBX_ERR_INVALID_ARGUMENT for a bad magic,
 * version or size, UBX_ERR_UNSUPPORTED for a dtype or geometry other than the
 * pool's (no conversion is done).
 */
int ubx_kv_wire_header_check(const ubx_kv_wire_header* header, int dtype, int num_layers, int num_kv_heads,
                             int head_dim, int block_size, uint64_t payload_bytes);

/*
 * Copy num_pages pages of num_layers layers (K and V) from one page layout to
 * another, on `stream` of the current device. Each side is either a pool --
 * base of KVPool.data, (num_layers, 2, num_blocks, block_size, num_kv_heads,
 * head_dim), element strides (s_layer, s_kv, s_block), page ids `pages` (int32
 * device array, entry i is the i-th page to copy) -- or, with pages == NULL, a
 * packed wire payload (page i at position i, strides (2 * num_pages *
 * page_elems, num_pages * page_elems, page_elems)).
 *   pool -> packed:  serialize (checksum: device uint64 that receives the
 *                    payload checksum of the header, or NULL)
 *   packed -> pool:  deserialize into the receiver's own page ids
 *   pool -> pool:    direct hand-off; dst may be another GPU's memory mapped
 *                    into this process (ubx_enable_peer_access, ubx_ipc_open_handle)
 * page_elems = block_size * num_kv_heads * head_dim; every base and stride a
 * multiple of 16 bytes. A page id outside [0, num_blocks) of its side skips
 * that page and sets UBX_DEVERR_BAD_PAGE in error_word (may be NULL).
 */
int ubx_kv_pages_copy(const void* src, int64_t src_s_layer, int64_t src_s_kv, int64_t src_s_block,
                      const int32_t* src_pages, int64_t src_num_blocks, void* dst, int64_t dst_s_layer,
                      int64_t dst_s_kv, int64_t dst_s_block, const int32_t* dst_pages, int64_t dst_num_blocks,
                      int num_layers, int num_pages, int64_t page_elems, int dtype, uint64_t* checksum,
                      int32_t* error_word, void* stream);

/* Let the current device read and write `peer_device`'s memory (no-op if already enabled). */
int ubx_enable_peer_access(int peer_device);
/*
 * CUDA IPC of a device buffer for a hand-off between worker processes:
 * ubx_ipc_get_handle writes the 64-byte handle of the allocation holding
 * dev_ptr and dev_ptr's offset inside it; ubx_ipc_open_handle maps it in
 * another process (peer access enabled) and returns the allocation's base
 * there (add the offset); ubx_ipc_close_handle unmaps it.
 */
int ubx_ipc_get_handle(const void* dev_ptr, void* handle_out, uint64_t* offset_out);
int ubx_ipc_open_handle(const void* handle, void** base_out);
int ubx_ipc_close_handle(void* base);

/*
 * Allocation-free variant of ubx_paged_decode_attention. No counterpart in the
 * reference: it exists for callers that cannot allocate device memory -- an
 * engine that gives all free HBM to its own KV pool at start-up and owns every
 * later allocation, or a binding from another language that holds only the
 * input and output buffers and no device allocator. Same arguments and results
 * as ubx_paged_decode_attention, minus the workspace: the scratch lives in a
 * fixed 8 MiB array inside the library (every GPU that loads the library holds
 * it until the process exits). Sizes whose scratch would exceed it are rejected
 * with UBX_ERR_WORKSPACE and a message naming the limit and the bytes the call
 * needs (on a 148-SM B200 the balanced schedule needs about 2.6 MiB in all at
 * 16 heads of 112; the split schedule needs roughly batch *
 * ceil(max_blocks_per_seq / split_pages) * num_heads * (4*head_dim + 8) bytes
 * beyond the 256 KiB counter prefix, plus 256-byte alignment of each region).
 * The call
 * itself allocates nothing.
 * The first call on each device looks up the array's device address (with that
 * device current) and caches it for the process; make that first call before
 * any stream capture. The device's primary context is assumed: after
 * cudaDeviceReset, or under another driver-API context, the cached address is
 * stale, so neither is supported. Every call shares the one array per device;
 * once its arguments pass every check it clears the counters and error word on
 * `stream` and launches (a rejected call touches nothing), so calls that
 * overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller.
 *   error_word: optional device int32 that receives the call's UBX_DEVERR_* bits.
 */
int ubx_paged_decode_attention_noalloc(const void* q, int64_t q_s_b, int64_t q_s_h, const void* k_cache,
                                       const void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                                       const int32_t* block_table, int64_t bt_s_row, const int32_t* context_lens,
                                       void* out, int64_t o_s_b, int64_t o_s_h, int batch, int num_heads,
                                       int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                                       int max_blocks_per_seq, float scale, int dtype, int schedule, int split_pages,
                                       int32_t* error_word, void* stream);

/*
 * Read (and optionally clear) the device error word of a workspace. This one
 * call synchronises `stream`.
 */
int ubx_read_device_error(const void* workspace, int32_t* value, int clear, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* UNBOX_B200_H_ */
