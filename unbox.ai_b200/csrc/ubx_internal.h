// Internal launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ubx {

constexpr int kBlockSize = 16;          // tokens per page (configs/infer/serve.yaml block_size)
constexpr int kMaxStages = 8;           // pipeline depth limit
constexpr int kStageSlotBytes = 2 * 8;  // per stage: full and empty mbarriers
constexpr int kMaxConsumerWarps = 8;    // consumer warps per CTA
constexpr int kMaxBatchSmem = 2048;     // balanced schedule keeps a (B+1) page prefix in smem
constexpr int kMaxTileBytes = 36864;    // one K (or V) page tile of a head group
constexpr int kSmemLimit = 227 * 1024 - 256;  // dynamic smem budget: 227 KB opt-in minus static smem (128 B)
constexpr int kSmemPerSm = 228 * 1024;        // shared memory of one SM
constexpr int kSmemReservedPerCta = 1024 + 512;  // per-CTA reservation + static smem
constexpr int kMaxCtasPerSm = 4;              // CTAs of one balanced launch per SM (small head groups)
constexpr int kCascadeFollowerSmem = 4096;     // per SM, left by the cascade's suffix pass to the merge CTAs
#ifndef UBX_TAIL_TRIM_PAGES
#define UBX_TAIL_TRIM_PAGES 4
#endif
// Balanced schedule under programmatic overlap, one CTA per SM: pages fewer
// for the last CTA, which starts only once the previous grid's last CTA has
// left its SM (the others start as their SMs free and prefetch meanwhile).
constexpr int kTailTrimPages = UBX_TAIL_TRIM_PAGES;

// Workspace layout prefix: [error word + reserved | merge counters | partials].
constexpr size_t kWsHeaderBytes = 256;                      // error word at offset 0
constexpr size_t kWsCounterEntries = 65536;                 // balanced-schedule merge counters
constexpr size_t kWsCounterBytes = kWsCounterEntries * 4;   // must be zero before a call
constexpr size_t kWsZeroBytes = kWsHeaderBytes + kWsCounterBytes;  // the prefix ubx_workspace_init zeroes

// Shared-memory row pitch of a page tile: one token row of the CTA's heads
// (heads * head_dim elements, contiguous in the KVPool layout) plus 16 bytes
// when needed to make the pitch an odd number of 16-byte chunks, so that the 8
// token rows one ldmatrix phase reads fall in 8 different bank groups.
constexpr int tile_row_pitch(int row_bytes) { return ((row_bytes / 16) & 1) ? row_bytes : row_bytes + 16; }

struct DecodeParams {
  const void* q;
  int64_t q_sb, q_sh;
  void* out;
  int64_t o_sb, o_sh;
  const int32_t* block_table;
  int64_t bt_sb;
  const int32_t* context_lens;
  int batch;
  int num_heads;
  int num_kv_heads;
  int max_blocks;
  int64_t num_blocks;
  float scale_log2;      // softmax scale * log2(e): scores live in the exp2 domain
  int tile_bytes;        // bytes of one K (or V) page tile in shared memory (16 rows)
  int row_bytes;         // bytes of one token row of the CTA's heads (one bulk copy)
  int smem_row_bytes;    // row pitch of a tile in shared memory
  int pbuf_bytes;        // bytes of the fp32 path's probability buffers
  int heads_per_cta;     // KV heads in one page tile (HG)
  int warps_per_kv;      // consumer warps sharing one KV head (WPK = G / GW)
  int stages;            // pipeline depth
  int split_pages;       // split schedule: pages per chunk
  int max_chunks;        // split schedule: chunk slots per sequence
  int tail_trim;         // balanced schedule: pages fewer for the last CTA's range (0: equal shares)
  int range_first;       // balanced schedule: first CTA of the page ranges (0; a fused cascade launch runs
                         // its shared-prefix CTAs below it)
  float* part_o;         // [slots][num_heads][D] unnormalised partial outputs
  float2* part_ml;       // [slots][num_heads] (running max in log2 units, denominator)
  int32_t* counters;     // [batch][num_kv_heads * warps_per_kv] merge counters (balanced)
  int32_t* error;        // device error word
  // raw pool views (fused append writes the new token's rows through them)
  const void* k_cache;
  const void* v_cache;
  int64_t c_sblk, c_stok, c_sh;
  // fused append (null when the call only attends): row t of k_new / v_new is
  // the token at position context_lens[t] - 1
  const void* k_new;
  const void* v_new;
  int64_t n_stok, n_sh;
  // fused pre-attention (null rope: q and k_new are used as given): RMSNorm with
  // q_w / k_w and the rotary embedding at position context_lens[b] - 1 are
  // applied to q and to the appended k row
  const void* q_w;
  const void* k_w;
  float eps;
  const float* rope;   // (rope_n, head_dim / 2) float2 (cos, sin)
  int64_t rope_sp;     // float stride between rope rows
  int rope_n;
  // optional (batch, num_heads) output: log2 of the softmax denominator in the
  // exp2 domain, m * scale * log2(e) + log2(sum), -inf for an empty context
  float* lse;
};

// Standalone pre-attention step (qk_norm_rope.cu); strides in elements.
struct PrepParams {
  const void* q_in;
  const void* k_in;
  const void* v_in;
  int64_t q_st, q_sh, k_st, k_sh, v_st, v_sh;
  const void* q_w;
  const void* k_w;
  float eps;
  const float* rope;
  int64_t rope_sp;
  int rope_n;
  const int32_t* positions;
  void* q_out;
  int64_t qo_st, qo_sh;
  void* k_out;  // may be null
  int64_t ko_st, ko_sh;
  void* k_cache;  // null: no append
  void* v_cache;
  int64_t c_sblk, c_stok, c_sh;
  const int64_t* slots;
  int64_t num_blocks;
  int block_size;
  int64_t num_tokens;
  int num_heads, num_kv_heads, head_dim;
  int32_t* error;
};

// Message returned by ubx_last_error() on this host thread (set by any entry point).
void set_last_error(const char* msg);
const char* last_error();

// ubx_paged_decode_attention that first zeroes the first `clear_bytes` of the
// workspace on `stream`, after every argument check has passed and right
// before the launch (capi.cu; the allocation-free entry point's shared scratch).
int paged_decode_attention_cleared(const void* q, int64_t q_s_b, int64_t q_s_h, const void* k_cache,
                                   const void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                                   const int32_t* block_table, int64_t bt_s_row, const int32_t* context_lens,
                                   void* out, int64_t o_s_b, int64_t o_s_h, int batch, int num_heads, int num_kv_heads,
                                   int head_dim, int block_size, int64_t num_blocks, int max_blocks_per_seq,
                                   float scale, int dtype, int schedule, int split_pages, void* workspace,
                                   size_t workspace_bytes, size_t clear_bytes, void* stream);

struct LaunchShape {
  dim3 grid;
  dim3 block;
  int smem_bytes;
  bool overlap;  // programmatic dependent launch on the previous kernel of the stream
};

// Shared-memory bytes the decode kernel needs (stage ring + softmax buffers +
// barriers + optional page prefix).
int decode_smem_bytes(int tile_bytes, int pbuf_bytes, int stages, int prefix_entries);

cudaError_t launch_paged_decode(int dtype, int head_dim, int gw, bool balanced, const DecodeParams& p,
                                const LaunchShape& shape, cudaStream_t stream);

cudaError_t launch_lse_combine(int dtype, int head_dim, const DecodeParams& p, cudaStream_t stream);

cudaError_t launch_kv_append(const void* k_new, const void* v_new, int64_t n_stok_b, int64_t n_sh_b, void* k_cache,
                             void* v_cache, int64_t c_sblk_b, int64_t c_stok_b, int64_t c_sh_b,
                             const int64_t* slots, int64_t num_tokens, int num_kv_heads, int row_bytes,
                             int block_size, int64_t num_blocks, int vec_bytes, int32_t* error_word,
                             cudaStream_t stream);
cudaError_t launch_prefill_append(const void* k_new, const void* v_new, int64_t n_stok_b, int64_t n_sh_b,
                                  void* k_cache, void* v_cache, int64_t c_sblk_b, int64_t c_stok_b, int64_t c_sh_b,
                                  const int32_t* bt_row, int max_blocks, int64_t start_pos, int64_t num_tokens,
                                  int num_kv_heads, int row_bytes, int block_size, int64_t num_blocks, int vec_bytes,
                                  int64_t* slots_out, int32_t* error_word, bool overlap, cudaStream_t stream);

cudaError_t launch_qk_norm_rope(int dtype, const PrepParams& p, cudaStream_t stream);

// Page copy between two page layouts (kv_transfer.cu); byte strides.
struct KvCopyParams {
  const void* src;
  int64_t src_s_layer, src_s_kv, src_s_block;
  const int32_t* src_pages;  // null: packed (page i at position i)
  int64_t src_num_blocks;
  void* dst;
  int64_t dst_s_layer, dst_s_kv, dst_s_block;
  const int32_t* dst_pages;
  int64_t dst_num_blocks;
  int num_layers, num_pages;
  int64_t page_bytes;
  unsigned long long* checksum;  // null: none
  int32_t* error;
  bool cross_gpu;  // source or destination outside this GPU's memory: plain loads and stores, no TMA
};

cudaError_t launch_kv_pages_copy(const KvCopyParams& p, cudaStream_t stream);

// Shared-prefix (cascade) pass (cascade.cu).
constexpr int kCascadeMaxPages = 8;      // shared pages of one chunk in shared memory (128 tokens)
constexpr int kCascadeMaxItemPages = 64; // shared pages of one work item (up to 8 chunks, one after another)
constexpr int kCascadeWorkInts = 6;      // ints per work item
constexpr int kCascadeRows = 128;        // (member, query head) rows of one work item: M of the MMAs
constexpr int kCascadeMinSmem = 80 * 1024;  // at most two prefix CTAs per SM

struct CascadeParams {
  // K and V pools as 3-D tensor maps (8 elements of a 16-byte chunk, the chunks
  // of every KV head's row, the tokens of every page): a box is one 16-byte
  // chunk column of one page (16 tokens), the layout of the operand tiles.
  // Filled, and use_tma set, when the driver encodes them.
  CUtensorMap tmap_k;
  CUtensorMap tmap_v;
  int use_tma;
  const void* q;
  int64_t q_sb, q_sh;
  const void* k_cache;
  const void* v_cache;
  int64_t c_sblk, c_stok;  // element strides; heads of a token row are contiguous
  int64_t num_blocks;
  const int32_t* page_list;    // shared page ids of every group, concatenated
  const int32_t* member_list;  // member sequences of every group, concatenated
  const int32_t* work;         // [num_work][6]: member offset, members, page offset, pages, chunk, 0
  int num_work;
  int batch, num_heads, num_kv_heads, max_chunks;
  float scale_log2;
  int pitch;                   // shared-memory row pitch (bytes) of one head row
  float* part_o;               // [batch][num_heads][max_chunks][D]
  float2* part_ml;             // [batch][num_heads][max_chunks] (max in log2 units, sum)
  int32_t* error;
  bool overlap;                // programmatic dependent launch; shared pages load before the wait
};

struct CascadeMergeParams {
  void* out;
  int64_t o_sb, o_sh;
  const float* lse;            // [batch][num_heads] of the suffix pass
  const int32_t* items;        // [num_items][2]: sequence, prefix chunks
  int num_items;
  int batch, num_heads, max_chunks;
  const float* part_o;
  const float2* part_ml;
  int32_t* error;
  bool overlap;                // programmatic dependent launch
};

int cascade_smem_bytes(int head_dim);
// One launch of a cascade step's suffix pass (DecodeParams, balanced schedule,
// CTAs from p.range_first on) and shared-prefix pass (CTAs below p.range_first);
// 16-bit pools, one CTA per SM (paged_decode.cu).
cudaError_t launch_cascade_fused(int dtype, int head_dim, const DecodeParams& p, const CascadeParams& cp,
                                 const LaunchShape& shape, cudaStream_t stream);
// Shared memory the prefix CTAs of that launch need (two pipelines of tiles).
int fused_prefix_smem_bytes(int head_dim);
cudaError_t launch_cascade_prefix(int dtype, int head_dim, const CascadeParams& p, cudaStream_t stream);
cudaError_t launch_cascade_merge(int dtype, int head_dim, const CascadeMergeParams& p, cudaStream_t stream);

cudaError_t launch_slot_mapping(const int32_t* block_table, int64_t bt_s_row, const int32_t* positions,
                                int64_t* slot_mapping, int batch, int max_blocks, int block_size,
                                cudaStream_t stream);

}  // namespace ubx
