// C ABI of unbox_b200: argument validation, launch planning, TMA descriptor
// encoding and the extern "C" entry points declared in include/unbox_b200.h.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "ubx_internal.h"
#include "../../include/unbox_b200.h"

namespace ubx {
namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(UBX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int dtype_bytes(int dtype) { return dtype == UBX_DTYPE_F32 ? 4 : 2; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- workspace layout (fixed prefix so that counters stay zero across calls)
constexpr size_t kHeaderBytes = kWsHeaderBytes;        // error word + reserved
constexpr size_t kCounterEntries = kWsCounterEntries;  // merge counters, re-armed by the kernel
constexpr int kDefaultSplitPages = 32;                 // 512-token split-KV chunks

// UBX_SCHEDULE_AUTO for a few long sequences: the balanced schedule cuts each
// of them over many CTAs, and the last part's warp merges every part (one
// sequence of 32k tokens: 148 parts, 92 us on a B200), while split-KV chunks of
// about (batch * max_blocks / SMs) pages, merged by the parallel combine
// kernel, take 31 us. Measured crossover (B200, GQA 16/8, head_dim 112, bf16):
// split wins for batch <= 4 with contexts of 8k-32k tokens (27-88 us against
// 42-96 us), ties at batch 6 and loses from batch 8 (157 against 168-176 us at
// 32k tokens) and on the 760M batch (54 against 74-88 us).
constexpr int kAutoSplitMaxBatch = 4;
constexpr int kAutoSplitMinBlocks = 64;

bool auto_prefers_split(int batch, int max_blocks) {
  return batch <= kAutoSplitMaxBatch && max_blocks >= kAutoSplitMinBlocks;
}

// Pages per chunk for the split schedule: the caller's choice, else about one
// wave of chunks (batch * max_blocks / SMs pages, a power of two in [16, 64])
// when AUTO picks split, else kDefaultSplitPages.
int split_pages_for(int split_pages, int schedule, int batch, int max_blocks, int num_sms) {
  if (split_pages > 0) return split_pages;
  if (schedule == UBX_SCHEDULE_AUTO && auto_prefers_split(batch, max_blocks)) {
    const int64_t want = ((int64_t)batch * max_blocks + num_sms - 1) / num_sms;
    int sp = 16;
    while (sp < want && sp < 64) sp *= 2;
    return sp;
  }
  return kDefaultSplitPages;
}
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct WsLayout {
  size_t ml_off, o_off, total;
  int64_t slots;
};

// [zeroed prefix | partials (max, sum) | partial outputs]
WsLayout ws_layout(int64_t slots, int num_heads, int head_dim) {
  WsLayout w;
  w.slots = slots;
  w.ml_off = kWsZeroBytes;
  w.o_off = w.ml_off + align256((size_t)slots * num_heads * sizeof(float2));
  w.total = w.o_off + (size_t)slots * num_heads * head_dim * sizeof(float);
  return w;
}

int num_sms_current_device(int* n) {
  static int cache[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev >= 0 && dev < 64 && cache[dev] > 0) {
    *n = cache[dev];
    return UBX_OK;
  }
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(MultiProcessorCount)");
  if (dev >= 0 && dev < 64) cache[dev] = sms;
  *n = sms;
  return UBX_OK;
}

struct Plan {
  int gw, wpk, hg, n_hg, stages, smem, row, pitch, tile, pbuf, ctas_per_sm;
  bool balanced;
  int split_pages, max_chunks;
  dim3 grid, block;
  int64_t slots;
};

// smem_reserve: shared memory per SM left to the small CTAs of the launches
// that follow (with programmatic overlap they become resident while this grid
// runs, and a CTA reserves 1 KB even with no shared memory of its own).
int make_plan(int batch, int num_heads, int num_kv_heads, int head_dim, int dtype, int max_blocks, int schedule,
              int split_pages, int num_sms, Plan* pl, int smem_reserve = 0) {
  const int G = num_heads / num_kv_heads;
  const int es = dtype_bytes(dtype);
  const bool mma = es == 2;  // 16-bit: tensor-core consumer, one warp per KV head
  pl->gw = mma ? G : (G < 2 ? G : 2);
  pl->wpk = mma ? 1 : G / pl->gw;
  pl->hg = 1;
  for (int hg = num_kv_heads; hg >= 1; --hg) {
    if (num_kv_heads % hg) continue;
    if (hg * pl->wpk > kMaxConsumerWarps) continue;
    if (kBlockSize * tile_row_pitch(hg * head_dim * es) > kMaxTileBytes) continue;
    pl->hg = hg;
    break;
  }
  pl->row = pl->hg * head_dim * es;      // one bulk copy: a token row of the CTA's heads
  pl->pitch = tile_row_pitch(pl->row);   // its shared-memory pitch
  pl->n_hg = num_kv_heads / pl->hg;
  const bool can_balance = batch <= kMaxBatchSmem && (int64_t)batch * num_kv_heads * pl->wpk <= (int64_t)kCounterEntries;
  if (schedule == UBX_SCHEDULE_BALANCED && !can_balance)
    return fail(UBX_ERR_UNSUPPORTED, "the balanced schedule needs batch <= %d (got %d)", kMaxBatchSmem, batch);
  pl->balanced = schedule == UBX_SCHEDULE_BALANCED ||
                 (schedule == UBX_SCHEDULE_AUTO && can_balance && !auto_prefers_split(batch, max_blocks));
  pl->split_pages = split_pages_for(split_pages, schedule, batch, max_blocks, num_sms);
  pl->max_chunks = (max_blocks + pl->split_pages - 1) / pl->split_pages;
  pl->tile = kBlockSize * pl->pitch;
  pl->pbuf = mma ? 0 : ((pl->hg * pl->wpk * pl->gw * kBlockSize * 4 + 15) & ~15);
  const int prefix = pl->balanced ? batch + 1 : 0;
  const int fixed = decode_smem_bytes(pl->tile, pl->pbuf, 0, prefix);
  // Small head groups leave a CTA with few consumer warps: put several CTAs on
  // an SM (aiming at 8 consumer warps per SM) and share its shared memory.
  const int ncw = pl->hg * pl->wpk;
  int ctas = std::min(kMaxCtasPerSm, (kMaxConsumerWarps + ncw - 1) / ncw);
  for (;; --ctas) {
    const int budget = (ctas == 1 ? kSmemLimit : kSmemPerSm / ctas - kSmemReservedPerCta) - smem_reserve / ctas;
    pl->stages = std::min(6, (budget - fixed) / (2 * pl->tile + kStageSlotBytes));
    if (pl->stages >= 2 || ctas == 1) break;
  }
  if (pl->stages < 2) return fail(UBX_ERR_UNSUPPORTED, "shared memory too small for a 2-stage pipeline");
  pl->ctas_per_sm = ctas;
  pl->smem = decode_smem_bytes(pl->tile, pl->pbuf, pl->stages, prefix);
  pl->block = dim3((pl->hg * pl->wpk + 1) * 32);
  if (pl->balanced) {
    pl->grid = dim3(std::max(1, num_sms * ctas / pl->n_hg), pl->n_hg);
    pl->slots = 2 * (int64_t)pl->grid.x;
  } else {
    pl->grid = dim3((unsigned)((int64_t)batch * pl->max_chunks), pl->n_hg);
    pl->slots = (int64_t)batch * pl->max_chunks;
  }
  return UBX_OK;
}

int check_shape(int num_heads, int num_kv_heads, int head_dim, int block_size, int dtype) {
  if (dtype != UBX_DTYPE_F32 && dtype != UBX_DTYPE_BF16 && dtype != UBX_DTYPE_F16)
    return fail(UBX_ERR_INVALID_ARGUMENT, "unknown dtype code %d", dtype);
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads)
    return fail(UBX_ERR_INVALID_ARGUMENT, "num_heads (%d) must be a positive multiple of num_kv_heads (%d)",
                num_heads, num_kv_heads);
  const int G = num_heads / num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return fail(UBX_ERR_UNSUPPORTED, "GQA ratio %d not built (1, 2, 4, 8)", G);
  if (head_dim != 64 && head_dim != 112 && head_dim != 128)
    return fail(UBX_ERR_UNSUPPORTED, "head_dim %d not built (64, 112, 128)", head_dim);
  if (block_size != kBlockSize) return fail(UBX_ERR_UNSUPPORTED, "block_size %d not built (16)", block_size);
  return UBX_OK;
}

}  // namespace

void set_last_error(const char* msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

}  // namespace ubx

using namespace ubx;

extern "C" {

const char* ubx_status_string(int status) {
  switch (status) {
    case UBX_OK: return "ok";
    case UBX_ERR_INVALID_ARGUMENT: return "invalid argument";
    case UBX_ERR_UNSUPPORTED: return "unsupported configuration";
    case UBX_ERR_WORKSPACE: return "workspace missing or too small";
    case UBX_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

const char* ubx_last_error(void) { return g_last_error.c_str(); }

int ubx_version(void) { return 100; }

int ubx_kv_append(const void* k_new, const void* v_new, int64_t new_s_tok, int64_t new_s_head, void* k_cache,
                  void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head, const int64_t* slot_mapping,
                  int64_t num_tokens, int num_kv_heads, int head_dim, int block_size, int64_t num_blocks, int dtype,
                  int32_t* error_word, void* stream) {
  g_last_error.clear();
  if (dtype != UBX_DTYPE_F32 && dtype != UBX_DTYPE_BF16 && dtype != UBX_DTYPE_F16)
    return fail(UBX_ERR_INVALID_ARGUMENT, "unknown dtype code %d", dtype);
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks <= 0)
    return fail(UBX_ERR_INVALID_ARGUMENT, "non-positive size");
  if (num_tokens == 0) return UBX_OK;
  if (!k_new || !v_new || !k_cache || !v_cache || !slot_mapping)
    return fail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  const int es = dtype_bytes(dtype);
  const int row = head_dim * es;
  // widest copy unit that every address and stride allows
  int vec = 16;
  auto ok_for = [&](int v) {
    auto a = [&](const void* p) { return (reinterpret_cast<uintptr_t>(p) % v) == 0; };
    auto s = [&](int64_t st) { return ((st * es) % v) == 0; };
    return row % v == 0 && a(k_new) && a(v_new) && a(k_cache) && a(v_cache) && s(new_s_tok) && s(new_s_head) &&
           s(c_s_block) && s(c_s_tok) && s(c_s_head);
  };
  while (vec > es && !ok_for(vec)) vec >>= 1;
  if (!ok_for(vec)) return fail(UBX_ERR_INVALID_ARGUMENT, "misaligned K/V row");
  cudaError_t e = launch_kv_append(k_new, v_new, new_s_tok * es, new_s_head * es, k_cache, v_cache, c_s_block * es,
                                   c_s_tok * es, c_s_head * es, slot_mapping, num_tokens, num_kv_heads, row,
                                   block_size, num_blocks, vec, error_word, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
  return UBX_OK;
}

int ubx_slot_mapping(const int32_t* block_table, int64_t bt_s_row, const int32_t* positions, int64_t* slot_mapping,
                     int batch, int max_blocks_per_seq, int block_size, void* stream) {
  g_last_error.clear();
  if (batch < 0 || block_size <= 0 || max_blocks_per_seq < 0) return fail(UBX_ERR_INVALID_ARGUMENT, "bad size");
  if (batch == 0) return UBX_OK;
  if (!block_table || !positions || !slot_mapping) return fail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  cudaError_t e = launch_slot_mapping(block_table, bt_s_row, positions, slot_mapping, batch, max_blocks_per_seq,
                                      block_size, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "slot_mapping launch");
  return UBX_OK;
}

int ubx_prefill_kv_write(const void* k, const void* v, int64_t s_tok, int64_t s_head, void* k_cache, void* v_cache,
                         int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head, const int32_t* block_table_row,
                         int max_blocks_per_seq, int64_t start_pos, int64_t num_tokens, int num_kv_heads, int head_dim,
                         int block_size, int64_t num_blocks, int dtype, int64_t* slots_out, int32_t* error_word,
                         int flags, void* stream) {
  g_last_error.clear();
  if (flags & ~UBX_FLAG_OVERLAP_PREVIOUS) return fail(UBX_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  if (dtype != UBX_DTYPE_F32 && dtype != UBX_DTYPE_BF16 && dtype != UBX_DTYPE_F16)
    return fail(UBX_ERR_INVALID_ARGUMENT, "unknown dtype code %d", dtype);
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks <= 0 ||
      max_blocks_per_seq < 0 || start_pos < 0)
    return fail(UBX_ERR_INVALID_ARGUMENT, "non-positive size or negative start position");
  if (num_tokens == 0) return UBX_OK;
  if (!k || !v || !k_cache || !v_cache || !block_table_row) return fail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  const int es = dtype_bytes(dtype);
  const int row = head_dim * es;
  int vec = 16;  // widest copy unit that every address and stride allows
  auto ok_for = [&](int w) {
    auto a = [&](const void* p) { return (reinterpret_cast<uintptr_t>(p) % w) == 0; };
    auto st = [&](int64_t x) { return ((x * es) % w) == 0; };
    return row % w == 0 && a(k) && a(v) && a(k_cache) && a(v_cache) && st(s_tok) && st(s_head) && st(c_s_block) &&
           st(c_s_tok) && st(c_s_head);
  };
  while (vec > es && !ok_for(vec)) vec >>= 1;
  if (!ok_for(vec)) return fail(UBX_ERR_INVALID_ARGUMENT, "misaligned K/V row");
  cudaError_t e = launch_prefill_append(k, v, s_tok * es, s_head * es, k_cache, v_cache, c_s_block * es, c_s_tok * es,
                                        c_s_head * es, block_table_row, max_blocks_per_seq, start_pos, num_tokens,
                                        num_kv_heads, row, block_size, num_blocks, vec, slots_out, error_word,
                                        (flags & UBX_FLAG_OVERLAP_PREVIOUS) != 0, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "prefill_kv_write launch");
  return UBX_OK;
}

int ubx_qk_norm_rope_append(const void* q_in, int64_t q_s_tok, int64_t q_s_head, const void* k_in, int64_t k_s_tok,
                            int64_t k_s_head, const void* v_in, int64_t v_s_tok, int64_t v_s_head,
                            const void* q_weight, const void* k_weight, float eps, const float* rope,
                            int64_t rope_s_pos, int rope_positions, const int32_t* positions, void* q_out,
                            int64_t qo_s_tok, int64_t qo_s_head, void* k_out, int64_t ko_s_tok, int64_t ko_s_head,
                            void* k_cache, void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                            const int64_t* slot_mapping, int64_t num_blocks, int block_size, int64_t num_tokens,
                            int num_heads, int num_kv_heads, int head_dim, int dtype, int32_t* error_word,
                            void* stream) {
  g_last_error.clear();
  if (dtype != UBX_DTYPE_F32 && dtype != UBX_DTYPE_BF16 && dtype != UBX_DTYPE_F16)
    return fail(UBX_ERR_INVALID_ARGUMENT, "unknown dtype code %d", dtype);
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0)
    return fail(UBX_ERR_INVALID_ARGUMENT, "bad token or head count");
  if (head_dim < 2 || head_dim > 256 || (head_dim & 1))
    return fail(UBX_ERR_UNSUPPORTED, "head_dim %d not built (even, <= 256)", head_dim);
  if (num_tokens == 0) return UBX_OK;
  if (!q_in || !k_in || !q_weight || !k_weight || !rope || !positions || !q_out)
    return fail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  if (rope_positions <= 0 || rope_s_pos < head_dim || (rope_s_pos & 1) || (reinterpret_cast<uintptr_t>(rope) & 7))
    return fail(UBX_ERR_INVALID_ARGUMENT, "rope table: %d rows, row stride %lld floats (even, >= %d), 8-byte aligned",
                rope_positions, (long long)rope_s_pos, head_dim);
  if (!(eps >= 0.f) || eps > 1e30f) return fail(UBX_ERR_INVALID_ARGUMENT, "eps must be finite, >= 0");
  const bool append = k_cache != nullptr;
  if (append && (!v_cache || !v_in || !slot_mapping || num_blocks <= 0 || block_size <= 0))
    return fail(UBX_ERR_INVALID_ARGUMENT, "append needs v_in, v_cache, slot_mapping and a positive pool size");
  const int es = dtype_bytes(dtype);
  const uintptr_t pa = 2u * (uintptr_t)es;  // element-pair alignment
  auto ap = [&](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % pa) == 0; };
  auto ev = [](int64_t st) { return (st & 1) == 0; };
  if (!ap(q_in) || !ap(k_in) || !ap(v_in) || !ap(q_weight) || !ap(k_weight) || !ap(q_out) || !ap(k_out) ||
      !ap(k_cache) || !ap(v_cache))
    return fail(UBX_ERR_INVALID_ARGUMENT, "rows must be aligned to element pairs (%d bytes)", (int)pa);
  if (!ev(q_s_tok) || !ev(q_s_head) || !ev(k_s_tok) || !ev(k_s_head) || !ev(qo_s_tok) || !ev(qo_s_head) ||
      (k_out && (!ev(ko_s_tok) || !ev(ko_s_head))) ||
      (append && (!ev(v_s_tok) || !ev(v_s_head) || !ev(c_s_block) || !ev(c_s_tok) || !ev(c_s_head))))
    return fail(UBX_ERR_INVALID_ARGUMENT, "strides must be even (element pairs)");
  PrepParams p;
  p.q_in = q_in;
  p.k_in = k_in;
  p.v_in = v_in;
  p.q_st = q_s_tok;
  p.q_sh = q_s_head;
  p.k_st = k_s_tok;
  p.k_sh = k_s_head;
  p.v_st = v_s_tok;
  p.v_sh = v_s_head;
  p.q_w = q_weight;
  p.k_w = k_weight;
  p.eps = eps;
  p.rope = rope;
  p.rope_sp = rope_s_pos;
  p.rope_n = rope_positions;
  p.positions = positions;
  p.q_out = q_out;
  p.qo_st = qo_s_tok;
  p.qo_sh = qo_s_head;
  p.k_out = k_out;
  p.ko_st = ko_s_tok;
  p.ko_sh = ko_s_head;
  p.k_cache = append ? k_cache : nullptr;
  p.v_cache = append ? v_cache : nullptr;
  p.c_sblk = c_s_block;
  p.c_stok = c_s_tok;
  p.c_sh = c_s_head;
  p.slots = slot_mapping;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.num_tokens = num_tokens;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.error = error_word;
  cudaError_t e = launch_qk_norm_rope(dtype, p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "qk_norm_rope launch");
  return UBX_OK;
}

int ubx_paged_decode_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim, int max_blocks_per_seq,
                                    int split_pages, int dtype, size_t* bytes) {
  g_last_error.clear();
  if (!bytes || batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || head_dim <= 0 ||
      max_blocks_per_seq < 0)
    return fail(UBX_ERR_INVALID_ARGUMENT, "bad workspace size query");
  int sms = 0;
  int st = num_sms_current_device(&sms);
  if (st != UBX_OK) return st;
  // room for the chunk size AUTO would pick too
  const int sp = std::min(split_pages_for(split_pages, UBX_SCHEDULE_AUTO, batch, max_blocks_per_seq, sms),
                          split_pages > 0 ? split_pages : kDefaultSplitPages);
  const int64_t chunks = (max_blocks_per_seq + sp - 1) / sp;
  const int64_t slots = std::max<int64_t>(2 * (int64_t)sms * kMaxCtasPerSm, (int64_t)batch * chunks);
  *bytes = ws_layout(slots, num_heads, head_dim).total;
  return UBX_OK;
}

int ubx_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (!workspace || workspace_bytes < kWsZeroBytes)
    return fail(UBX_ERR_WORKSPACE, "workspace smaller than its fixed header (%zu bytes)", kWsZeroBytes);
  cudaError_t e = cudaMemsetAsync(workspace, 0, kWsZeroBytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "workspace memset");
  return UBX_OK;
}

int ubx_read_device_error(const void* workspace, int32_t* value, int clear, void* stream) {
  g_last_error.clear();
  if (!workspace || !value) return fail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(value, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(const_cast<void*>(workspace), 0, sizeof(int32_t), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "read device error word");
  return UBX_OK;
}

}  // extern "C"

namespace {

struct AppendArgs {
  const void* k_new;
  const void* v_new;
  int64_t s_tok, s_head;  // element strides of k_new / v_new
};

struct PrepArgs {
  const void* q_w;
  const void* k_w;
  float eps;
  const float* rope;
  int64_t rope_sp;
  int rope_n;
};

int decode_impl(const void* q, int64_t q_s_b, int64_t q_s_h, const void* k_cache, const void* v_cache,
                int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head, const int32_t* block_table, int64_t bt_s_row,
                const int32_t* context_lens, void* out, int64_t o_s_b, int64_t o_s_h, int batch, int num_heads,
                int num_kv_heads, int head_dim, int block_size, int64_t num_blocks, int max_blocks_per_seq,
                float scale, int dtype, int schedule, int split_pages, int flags, void* workspace,
                size_t workspace_bytes, const AppendArgs* app, const PrepArgs* prep, float* lse, void* stream,
                size_t clear_bytes = 0, CascadeParams* fuse = nullptr, int prefix_ctas = 0) {
  g_last_error.clear();
  int st = check_shape(num_heads, num_kv_heads, head_dim, block_size, dtype);
  if (st != UBX_OK) return st;
  if (batch < 0) return fail(UBX_ERR_INVALID_ARGUMENT, "negative batch");
  if (batch == 0) return UBX_OK;
  if (schedule != UBX_SCHEDULE_AUTO && schedule != UBX_SCHEDULE_BALANCED && schedule != UBX_SCHEDULE_SPLIT)
    return fail(UBX_ERR_INVALID_ARGUMENT, "unknown schedule %d", schedule);
  if (!q || !k_cache || !v_cache || !block_table || !context_lens || !out)
    return fail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  if (num_blocks <= 0 || num_blocks > (int64_t)0x7fffffff)
    return fail(UBX_ERR_INVALID_ARGUMENT, "num_blocks %lld out of range", (long long)num_blocks);
  if (max_blocks_per_seq <= 0) return fail(UBX_ERR_INVALID_ARGUMENT, "max_blocks_per_seq must be positive");
  const int es = dtype_bytes(dtype);
  auto m16 = [&](int64_t s) { return ((s * es) & 15) == 0; };
  if (!aligned16(q) || !aligned16(out) || !m16(q_s_b) || !m16(q_s_h) || !m16(o_s_b) || !m16(o_s_h))
    return fail(UBX_ERR_INVALID_ARGUMENT, "q/out rows must be 16-byte aligned");
  if (!aligned16(k_cache) || !aligned16(v_cache) || !m16(c_s_block) || !m16(c_s_tok) || !m16(c_s_head))
    return fail(UBX_ERR_INVALID_ARGUMENT, "K/V cache base and strides must be multiples of 16 bytes");
  if (c_s_head != head_dim)
    return fail(UBX_ERR_UNSUPPORTED,
                "KV heads must be contiguous within a token row (head stride %lld, head_dim %d): the KVPool layout",
                (long long)c_s_head, head_dim);
  if (app) {
    if (!app->k_new || !app->v_new) return fail(UBX_ERR_INVALID_ARGUMENT, "null k_new / v_new");
    if (!aligned16(app->k_new) || !aligned16(app->v_new) || !m16(app->s_tok) || !m16(app->s_head))
      return fail(UBX_ERR_INVALID_ARGUMENT, "k_new / v_new rows must be 16-byte aligned");
  }
  if (lse && es != 2)
    return fail(UBX_ERR_UNSUPPORTED, "the log-sum-exp output is built for bf16/f16");
  if (prep) {
    if (es != 2)
      return fail(UBX_ERR_UNSUPPORTED, "fused pre-attention is built for bf16/f16 (fp32: ubx_qk_norm_rope_append, "
                                       "then ubx_paged_decode_attention)");
    if (!prep->q_w || !prep->k_w || !prep->rope) return fail(UBX_ERR_INVALID_ARGUMENT, "null norm weight or rope table");
    if (!aligned16(prep->q_w) || !aligned16(prep->k_w) || !aligned16(prep->rope) || (prep->rope_sp & 3))
      return fail(UBX_ERR_INVALID_ARGUMENT, "norm weights and rope rows must be 16-byte aligned");
    if (prep->rope_n <= 0 || prep->rope_sp < head_dim)
      return fail(UBX_ERR_INVALID_ARGUMENT, "rope table of %d rows with row stride %lld floats (need >= %d)",
                  prep->rope_n, (long long)prep->rope_sp, head_dim);
    if (!(prep->eps >= 0.f) || prep->eps > 1e30f) return fail(UBX_ERR_INVALID_ARGUMENT, "eps must be finite, >= 0");
  }
  if (!(scale > 0.f) && !(scale < 0.f)) return fail(UBX_ERR_INVALID_ARGUMENT, "scale must be finite and non-zero");
  if (flags & ~UBX_FLAG_OVERLAP_PREVIOUS) return fail(UBX_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  if (!workspace) return fail(UBX_ERR_WORKSPACE, "workspace is required");
  if (!aligned16(workspace)) return fail(UBX_ERR_WORKSPACE, "workspace must be 16-byte aligned");

  int sms = 0;
  st = num_sms_current_device(&sms);
  if (st != UBX_OK) return st;
  // The log-sum-exp variant is the cascade's suffix pass: when its prefix and
  // merge launches follow with programmatic overlap, leave their CTAs room (the
  // one-launch step keeps every stage: only the merge follows it).
  const int reserve = (lse && !(fuse && prefix_ctas > 0)) ? kCascadeFollowerSmem : 0;
  Plan pl;
  st = make_plan(batch, num_heads, num_kv_heads, head_dim, dtype, max_blocks_per_seq, schedule, split_pages, sms, &pl,
                 reserve);
  if (st != UBX_OK) return st;
  const WsLayout wl = ws_layout(pl.slots, num_heads, head_dim);
  if (workspace_bytes < wl.total)
    return fail(UBX_ERR_WORKSPACE, "workspace of %zu bytes, this call needs %zu", workspace_bytes, wl.total);

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  DecodeParams p;
  p.q = q;
  p.q_sb = q_s_b;
  p.q_sh = q_s_h;
  p.out = out;
  p.o_sb = o_s_b;
  p.o_sh = o_s_h;
  p.block_table = block_table;
  p.bt_sb = bt_s_row;
  p.context_lens = context_lens;
  p.batch = batch;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.max_blocks = max_blocks_per_seq;
  p.num_blocks = num_blocks;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.tile_bytes = pl.tile;
  p.row_bytes = pl.row;
  p.smem_row_bytes = pl.pitch;
  p.pbuf_bytes = pl.pbuf;
  p.heads_per_cta = pl.hg;
  p.warps_per_kv = pl.wpk;
  p.stages = pl.stages;
  p.split_pages = pl.split_pages;
  p.max_chunks = pl.max_chunks;
  p.tail_trim = ((flags & UBX_FLAG_OVERLAP_PREVIOUS) && pl.balanced && pl.ctas_per_sm == 1 &&
                 pl.grid.y == 1)
                    ? kTailTrimPages : 0;
  p.range_first = 0;
  p.part_o = reinterpret_cast<float*>(ws + wl.o_off);
  p.part_ml = reinterpret_cast<float2*>(ws + wl.ml_off);
  p.counters = reinterpret_cast<int32_t*>(ws + kHeaderBytes);
  p.error = reinterpret_cast<int32_t*>(ws);
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.c_sblk = c_s_block;
  p.c_stok = c_s_tok;
  p.c_sh = c_s_head;
  p.k_new = app ? app->k_new : nullptr;
  p.v_new = app ? app->v_new : nullptr;
  p.n_stok = app ? app->s_tok : 0;
  p.n_sh = app ? app->s_head : 0;
  p.q_w = prep ? prep->q_w : nullptr;
  p.k_w = prep ? prep->k_w : nullptr;
  p.eps = prep ? prep->eps : 0.f;
  p.rope = prep ? prep->rope : nullptr;
  p.rope_sp = prep ? prep->rope_sp : 0;
  p.rope_n = prep ? prep->rope_n : 0;
  p.lse = lse;

  LaunchShape shape{pl.grid, pl.block, pl.smem, (flags & UBX_FLAG_OVERLAP_PREVIOUS) != 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (clear_bytes > 0) {
    // a workspace shared between calls (the allocation-free entry point) is
    // cleared only once the call has passed every check, so a rejected call
    // leaves the state of a call still running elsewhere alone
    cudaError_t ce = cudaMemsetAsync(workspace, 0, std::min(clear_bytes, workspace_bytes), s);
    if (ce != cudaSuccess) return cuda_fail(ce, "workspace clear");
  }
  if (fuse) {
    // a cascade step: the shared-prefix pass shares the launch when the suffix
    // pass runs one balanced CTA per SM (prefix CTAs first, on their own SMs);
    // otherwise it follows as its own launch
    fuse->error = p.error;
    const int fused_smem = std::max(pl.smem, fused_prefix_smem_bytes(head_dim));
    const bool fusable = pl.balanced && pl.ctas_per_sm == 1 && pl.grid.y == 1 && pl.grid.x >= 2 &&
                         dtype != UBX_DTYPE_F32 && fused_smem <= kSmemLimit;
    if (fusable && fuse->num_work > 0 && prefix_ctas > 0) {
      p.range_first = std::min(std::max(prefix_ctas, 1), (int)pl.grid.x - 1);
      LaunchShape fshape = shape;
      fshape.smem_bytes = fused_smem;
      cudaError_t e = launch_cascade_fused(dtype, head_dim, p, *fuse, fshape, s);
      if (e != cudaSuccess) return cuda_fail(e, "cascade launch");
      return UBX_OK;
    }
    cudaError_t e = launch_paged_decode(dtype, head_dim, pl.gw, pl.balanced, p, shape, s);
    if (e != cudaSuccess) return cuda_fail(e, "paged_decode launch");
    if (!pl.balanced) {
      e = launch_lse_combine(dtype, head_dim, p, s);
      if (e != cudaSuccess) return cuda_fail(e, "lse_combine launch");
    }
    fuse->overlap = true;  // follows a kernel of this call
    e = launch_cascade_prefix(dtype, head_dim, *fuse, s);
    if (e != cudaSuccess) return cuda_fail(e, "cascade prefix launch");
    return UBX_OK;
  }
  cudaError_t e = launch_paged_decode(dtype, head_dim, pl.gw, pl.balanced, p, shape, s);
  if (e != cudaSuccess) return cuda_fail(e, "paged_decode launch");
  if (!pl.balanced) {
    e = launch_lse_combine(dtype, head_dim, p, s);
    if (e != cudaSuccess) return cuda_fail(e, "lse_combine launch");
  }
  return UBX_OK;
}

}  // namespace

namespace ubx {

int paged_decode_attention_cleared(const void* q, int64_t q_s_b, int64_t q_s_h, const void* k_cache,
                                   const void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                                   const int32_t* block_table, int64_t bt_s_row, const int32_t* context_lens,
                                   void* out, int64_t o_s_b, int64_t o_s_h, int batch, int num_heads, int num_kv_heads,
                                   int head_dim, int block_size, int64_t num_blocks, int max_blocks_per_seq,
                                   float scale, int dtype, int schedule, int split_pages, void* workspace,
                                   size_t workspace_bytes, size_t clear_bytes, void* stream) {
  return decode_impl(q, q_s_b, q_s_h, k_cache, v_cache, c_s_block, c_s_tok, c_s_head, block_table, bt_s_row,
                     context_lens, out, o_s_b, o_s_h, batch, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                     max_blocks_per_seq, scale, dtype, schedule, split_pages, 0, workspace, workspace_bytes, nullptr,
                     nullptr, nullptr, stream, clear_bytes);
}

}  // namespace ubx

extern "C" {

int ubx_paged_decode_attention(const void* q, int64_t q_s_b, int64_t q_s_h, const void* k_cache, const void* v_cache,
                               int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head, const int32_t* block_table,
                               int64_t bt_s_row, const int32_t* context_lens, void* out, int64_t o_s_b, int64_t o_s_h,
                               int batch, int num_heads, int num_kv_heads, int head_dim, int block_size,
                               int64_t num_blocks, int max_blocks_per_seq, float scale, int dtype, int schedule,
                               int split_pages, void* workspace, size_t workspace_bytes, void* stream) {
  return decode_impl(q, q_s_b, q_s_h, k_cache, v_cache, c_s_block, c_s_tok, c_s_head, block_table, bt_s_row,
                     context_lens, out, o_s_b, o_s_h, batch, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                     max_blocks_per_seq, scale, dtype, schedule, split_pages, 0, workspace, workspace_bytes, nullptr,
                     nullptr, nullptr, stream);
}

int ubx_paged_decode_append_attention(const void* k_new, const void* v_new, int64_t new_s_tok, int64_t new_s_head,
                                      const void* q, int64_t q_s_b, int64_t q_s_h, void* k_cache, void* v_cache,
                                      int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                                      const int32_t* block_table, int64_t bt_s_row, const int32_t* context_lens,
                                      void* out, int64_t o_s_b, int64_t o_s_h, int batch, int num_heads,
                                      int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                                      int max_blocks_per_seq, float scale, int dtype, int schedule, int split_pages,
                                      int flags, void* workspace, size_t workspace_bytes, void* stream) {
  const AppendArgs app{k_new, v_new, new_s_tok, new_s_head};
  return decode_impl(q, q_s_b, q_s_h, k_cache, v_cache, c_s_block, c_s_tok, c_s_head, block_table, bt_s_row,
                     context_lens, out, o_s_b, o_s_h, batch, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                     max_blocks_per_seq, scale, dtype, schedule, split_pages, flags, workspace, workspace_bytes, &app,
                     nullptr, nullptr, stream);
}

int ubx_paged_decode_attention_lse(const void* k_new, const void* v_new, int64_t new_s_tok, int64_t new_s_head,
                                   const void* q, int64_t q_s_b, int64_t q_s_h, void* k_cache, void* v_cache,
                                   int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head, const int32_t* block_table,
                                   int64_t bt_s_row, const int32_t* context_lens, void* out, int64_t o_s_b,
                                   int64_t o_s_h, int batch, int num_heads, int num_kv_heads, int head_dim,
                                   int block_size, int64_t num_blocks, int max_blocks_per_seq, float scale, int dtype,
                                   int schedule, int split_pages, int flags, float* lse_out, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  if ((k_new == nullptr) != (v_new == nullptr)) {
    g_last_error = "pass both k_new and v_new, or neither";
    return UBX_ERR_INVALID_ARGUMENT;
  }
  if (!lse_out) {
    g_last_error = "lse_out is required";
    return UBX_ERR_INVALID_ARGUMENT;
  }
  const AppendArgs app{k_new, v_new, new_s_tok, new_s_head};
  return decode_impl(q, q_s_b, q_s_h, k_cache, v_cache, c_s_block, c_s_tok, c_s_head, block_table, bt_s_row,
                     context_lens, out, o_s_b, o_s_h, batch, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                     max_blocks_per_seq, scale, dtype, schedule, split_pages, flags, workspace, workspace_bytes,
                     k_new ? &app : nullptr, nullptr, lse_out, stream);
}

static size_t cascade_ml_bytes(int batch, int num_heads, int max_chunks) {
  return align256((size_t)batch * num_heads * max_chunks * sizeof(float2));
}

int ubx_cascade_workspace_size(int batch, int num_heads, int head_dim, int max_chunks, size_t* bytes) {
  g_last_error.clear();
  if (!bytes || batch < 0 || num_heads <= 0 || head_dim <= 0 || max_chunks < 0)
    return fail(UBX_ERR_INVALID_ARGUMENT, "bad cascade workspace query");
  *bytes = cascade_ml_bytes(batch, num_heads, max_chunks) +
           (size_t)batch * num_heads * max_chunks * head_dim * sizeof(float);
  return UBX_OK;
}

}  // extern "C"

namespace {

// A K or V pool as the prefix pass's 3-D tensor map: dimension 0 = the 8
// elements of a 16-byte chunk, 1 = the chunks of all KV heads' rows (16 bytes
// apart: heads are contiguous within a token row), 2 = every token of every
// page (c_s_tok elements apart); box = one chunk column of one page. Returns
// false when the driver's encoder is missing or refuses the layout (the pass
// then copies with cp.async).
bool encode_prefix_map(CUtensorMap* map, const void* pool, int dtype, int64_t num_blocks, int num_kv_heads,
                       int head_dim, int64_t c_s_tok) {
  using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode fn = nullptr;
  static bool looked = false;
  if (!looked) {
    looked = true;
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && f)
      fn = reinterpret_cast<Encode>(f);
  }
  if (!fn) return false;
  // the decode loop asks for the same pools every step: remember the last maps
  struct Entry {
    const void* pool;
    int dtype, kv_heads, head_dim;
    int64_t num_blocks, c_s_tok;
    CUtensorMap map;
  };
  static thread_local Entry cache[64];
  static thread_local int cache_n = 0, cache_next = 0;
  for (int i = 0; i < cache_n; ++i) {
    const Entry& c = cache[i];
    if (c.pool == pool && c.dtype == dtype && c.kv_heads == num_kv_heads && c.head_dim == head_dim &&
        c.num_blocks == num_blocks && c.c_s_tok == c_s_tok) {
      *map = c.map;
      return true;
    }
  }
  const cuuint64_t dims[3] = {8, (cuuint64_t)num_kv_heads * head_dim / 8, (cuuint64_t)num_blocks * kBlockSize};
  const cuuint64_t strides[2] = {16, (cuuint64_t)c_s_tok * 2};  // bytes, dimensions 1 and 2
  const cuuint32_t box[3] = {8, 1, (cuuint32_t)kBlockSize};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, dtype == UBX_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        3, const_cast<void*>(pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  cache[cache_next] = Entry{pool, dtype, num_kv_heads, head_dim, num_blocks, c_s_tok, *map};
  cache_next = (cache_next + 1) % 64;
  if (cache_n < 64) ++cache_n;
  return true;
}

// Checks the shared-prefix pass's arguments and fills its launch parameters
// (error word and overlap flag left to the caller).
int make_cascade_params(const void* q, int64_t q_s_b, int64_t q_s_h, const void* k_cache, const void* v_cache,
                        int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head, int64_t num_blocks,
                        const int32_t* page_list, const int32_t* member_list, const int32_t* work_items,
                        int num_work_items, int max_chunks, int batch, int num_heads, int num_kv_heads, int head_dim,
                        float scale, int dtype, void* cascade_ws, size_t cascade_ws_bytes, CascadeParams* out) {
  int st = check_shape(num_heads, num_kv_heads, head_dim, kBlockSize, dtype);
  if (st != UBX_OK) return st;
  if (dtype == UBX_DTYPE_F32) return fail(UBX_ERR_UNSUPPORTED, "the cascade pass is built for bf16/f16");
  if (num_work_items < 0 || max_chunks <= 0 || batch <= 0 || num_blocks <= 0)
    return fail(UBX_ERR_INVALID_ARGUMENT, "bad cascade sizes");
  if (num_work_items == 0) return UBX_OK;  // nothing to launch: *out is not used
  if (!q || !k_cache || !v_cache || !page_list || !member_list || !work_items || !cascade_ws)
    return fail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  const int es = 2;
  auto m16 = [&](int64_t s) { return ((s * es) & 15) == 0; };
  if (!aligned16(q) || !m16(q_s_b) || !m16(q_s_h) || !aligned16(k_cache) || !aligned16(v_cache) ||
      !m16(c_s_block) || !m16(c_s_tok))
    return fail(UBX_ERR_INVALID_ARGUMENT, "q rows and K/V caches must be 16-byte aligned");
  if (c_s_head != head_dim) return fail(UBX_ERR_UNSUPPORTED, "KV heads must be contiguous within a token row");
  size_t need = 0;
  ubx_cascade_workspace_size(batch, num_heads, head_dim, max_chunks, &need);
  if (cascade_ws_bytes < need)
    return fail(UBX_ERR_WORKSPACE, "cascade workspace of %zu bytes, this call needs %zu", cascade_ws_bytes, need);
  if (!aligned16(cascade_ws)) return fail(UBX_ERR_WORKSPACE, "cascade workspace must be 16-byte aligned");
  if (!(scale > 0.f) && !(scale < 0.f)) return fail(UBX_ERR_INVALID_ARGUMENT, "scale must be finite and non-zero");
  CascadeParams& p = *out;
  p.q = q;
  p.q_sb = q_s_b;
  p.q_sh = q_s_h;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.c_sblk = c_s_block;
  p.c_stok = c_s_tok;
  p.num_blocks = num_blocks;
  p.page_list = page_list;
  p.member_list = member_list;
  p.work = work_items;
  p.num_work = num_work_items;
  p.batch = batch;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.max_chunks = max_chunks;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.pitch = tile_row_pitch(head_dim * es);
  uint8_t* ws = static_cast<uint8_t*>(cascade_ws);
  p.part_ml = reinterpret_cast<float2*>(ws);
  p.part_o = reinterpret_cast<float*>(ws + cascade_ml_bytes(batch, num_heads, max_chunks));
  p.error = nullptr;
  p.overlap = false;
  // the tensor maps address token t of page g as row 16 g + t at one stride:
  // packed pages only (a padded or interleaved pool copies with cp.async)
  p.use_tma = c_s_block == (int64_t)kBlockSize * c_s_tok &&
              encode_prefix_map(&p.tmap_k, k_cache, dtype, num_blocks, num_kv_heads, head_dim, c_s_tok) &&
              encode_prefix_map(&p.tmap_v, v_cache, dtype, num_blocks, num_kv_heads, head_dim, c_s_tok);
  return UBX_OK;
}

}  // namespace

extern "C" {

int ubx_cascade_prefix_attention(const void* q, int64_t q_s_b, int64_t q_s_h, const void* k_cache,
                                 const void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                                 int64_t num_blocks, const int32_t* page_list, const int32_t* member_list,
                                 const int32_t* work_items, int num_work_items, int max_chunks, int batch,
                                 int num_heads, int num_kv_heads, int head_dim, float scale, int dtype,
                                 void* cascade_ws, size_t cascade_ws_bytes, int32_t* error_word, int flags,
                                 void* stream) {
  g_last_error.clear();
  if (flags & ~UBX_FLAG_OVERLAP_PREVIOUS) return fail(UBX_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  CascadeParams p;
  int st = make_cascade_params(q, q_s_b, q_s_h, k_cache, v_cache, c_s_block, c_s_tok, c_s_head, num_blocks,
                               page_list, member_list, work_items, num_work_items, max_chunks, batch, num_heads,
                               num_kv_heads, head_dim, scale, dtype, cascade_ws, cascade_ws_bytes, &p);
  if (st != UBX_OK || num_work_items == 0) return st;
  p.error = error_word;
  p.overlap = (flags & UBX_FLAG_OVERLAP_PREVIOUS) != 0;
  cudaError_t e = launch_cascade_prefix(dtype, head_dim, p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cascade prefix launch");
  return UBX_OK;
}

int ubx_cascade_merge(void* out, int64_t o_s_b, int64_t o_s_h, const float* lse, const int32_t* merge_items,
                      int num_merge_items, int max_chunks, int batch, int num_heads, int head_dim, int dtype,
                      const void* cascade_ws, size_t cascade_ws_bytes, int32_t* error_word, int flags,
                      void* stream) {
  g_last_error.clear();
  if (flags & ~UBX_FLAG_OVERLAP_PREVIOUS) return fail(UBX_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  if (dtype != UBX_DTYPE_BF16 && dtype != UBX_DTYPE_F16)
    return fail(UBX_ERR_UNSUPPORTED, "the cascade merge is built for bf16/f16");
  if (head_dim != 64 && head_dim != 112 && head_dim != 128)
    return fail(UBX_ERR_UNSUPPORTED, "head_dim %d not built (64, 112, 128)", head_dim);
  if (num_merge_items < 0 || max_chunks <= 0 || batch <= 0 || num_heads <= 0)
    return fail(UBX_ERR_INVALID_ARGUMENT, "bad merge sizes");
  if (num_merge_items == 0) return UBX_OK;
  if (!out || !lse || !merge_items || !cascade_ws) return fail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  auto m16 = [&](int64_t s) { return ((s * 2) & 15) == 0; };
  if (!aligned16(out) || !m16(o_s_b) || !m16(o_s_h)) return fail(UBX_ERR_INVALID_ARGUMENT, "out rows must be 16-byte aligned");
  size_t need = 0;
  ubx_cascade_workspace_size(batch, num_heads, head_dim, max_chunks, &need);
  if (cascade_ws_bytes < need)
    return fail(UBX_ERR_WORKSPACE, "cascade workspace of %zu bytes, this call needs %zu", cascade_ws_bytes, need);
  if (!aligned16(cascade_ws)) return fail(UBX_ERR_WORKSPACE, "cascade workspace must be 16-byte aligned");
  CascadeMergeParams p;
  p.out = out;
  p.o_sb = o_s_b;
  p.o_sh = o_s_h;
  p.lse = lse;
  p.items = merge_items;
  p.num_items = num_merge_items;
  p.batch = batch;
  p.num_heads = num_heads;
  p.max_chunks = max_chunks;
  const uint8_t* ws = static_cast<const uint8_t*>(cascade_ws);
  p.part_ml = reinterpret_cast<const float2*>(ws);
  p.part_o = reinterpret_cast<const float*>(ws + cascade_ml_bytes(batch, num_heads, max_chunks));
  p.error = error_word;
  p.overlap = (flags & UBX_FLAG_OVERLAP_PREVIOUS) != 0;
  cudaError_t e = launch_cascade_merge(dtype, head_dim, p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cascade merge launch");
  return UBX_OK;
}

int ubx_cascade_attention(const void* k_new, const void* v_new, int64_t new_s_tok, int64_t new_s_head,
                          const void* q, int64_t q_s_b, int64_t q_s_h, void* k_cache, void* v_cache,
                          int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head, const int32_t* suffix_block_table,
                          int64_t bt_s_row, const int32_t* suffix_context_lens, void* out, int64_t o_s_b,
                          int64_t o_s_h, int batch, int num_heads, int num_kv_heads, int head_dim, int block_size,
                          int64_t num_blocks, int max_blocks_per_seq, float scale, int dtype, int schedule,
                          const int32_t* page_list, const int32_t* member_list, const int32_t* work_items,
                          int num_work_items, const int32_t* merge_items, int num_merge_items, int max_chunks,
                          int prefix_ctas, int flags, float* lse_out, void* workspace, size_t workspace_bytes,
                          void* cascade_ws, size_t cascade_ws_bytes, void* stream) {
  g_last_error.clear();
  if ((k_new == nullptr) != (v_new == nullptr)) return fail(UBX_ERR_INVALID_ARGUMENT, "pass both k_new and v_new, or neither");
  if (!lse_out) return fail(UBX_ERR_INVALID_ARGUMENT, "lse_out is required");
  if (flags & ~UBX_FLAG_OVERLAP_PREVIOUS) return fail(UBX_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  if (dtype == UBX_DTYPE_F32) return fail(UBX_ERR_UNSUPPORTED, "the cascade is built for bf16/f16");
  if (num_merge_items < 0 || prefix_ctas < 0) return fail(UBX_ERR_INVALID_ARGUMENT, "bad cascade sizes");
  if (batch == 0) return UBX_OK;
  CascadeParams cp;
  int st = make_cascade_params(q, q_s_b, q_s_h, k_cache, v_cache, c_s_block, c_s_tok, c_s_head, num_blocks,
                               page_list, member_list, work_items, num_work_items, max_chunks, batch, num_heads,
                               num_kv_heads, head_dim, scale, dtype, cascade_ws, cascade_ws_bytes, &cp);
  if (st != UBX_OK) return st;
  if (num_merge_items > 0 && !merge_items) return fail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  const AppendArgs app{k_new, v_new, new_s_tok, new_s_head};
  st = decode_impl(q, q_s_b, q_s_h, k_cache, v_cache, c_s_block, c_s_tok, c_s_head, suffix_block_table, bt_s_row,
                   suffix_context_lens, out, o_s_b, o_s_h, batch, num_heads, num_kv_heads, head_dim, block_size,
                   num_blocks, max_blocks_per_seq, scale, dtype, schedule, 0, flags, workspace,
                   workspace_bytes, k_new ? &app : nullptr, nullptr, lse_out, stream, 0,
                   num_work_items > 0 ? &cp : nullptr, prefix_ctas);
  if (st != UBX_OK || num_work_items == 0 || num_merge_items == 0) return st;
  return ubx_cascade_merge(out, o_s_b, o_s_h, lse_out, merge_items, num_merge_items, max_chunks, batch, num_heads,
                           head_dim, dtype, cascade_ws, cascade_ws_bytes, static_cast<int32_t*>(workspace),
                           UBX_FLAG_OVERLAP_PREVIOUS, stream);
}

int ubx_paged_decode_prep_attention(const void* q_raw, int64_t q_s_b, int64_t q_s_h, const void* k_raw,
                                    const void* v_new, int64_t new_s_tok, int64_t new_s_head, const void* q_weight,
                                    const void* k_weight, float eps, const float* rope, int64_t rope_s_pos,
                                    int rope_positions, void* k_cache, void* v_cache, int64_t c_s_block,
                                    int64_t c_s_tok, int64_t c_s_head, const int32_t* block_table, int64_t bt_s_row,
                                    const int32_t* context_lens, void* out, int64_t o_s_b, int64_t o_s_h, int batch,
                                    int num_heads, int num_kv_heads, int head_dim, int block_size,
                                    int64_t num_blocks, int max_blocks_per_seq, float scale, int dtype, int schedule,
                                    int split_pages, int flags, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  const AppendArgs app{k_raw, v_new, new_s_tok, new_s_head};
  const PrepArgs prep{q_weight, k_weight, eps, rope, rope_s_pos, rope_positions};
  return decode_impl(q_raw, q_s_b, q_s_h, k_cache, v_cache, c_s_block, c_s_tok, c_s_head, block_table, bt_s_row,
                     context_lens, out, o_s_b, o_s_h, batch, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                     max_blocks_per_seq, scale, dtype, schedule, split_pages, flags, workspace, workspace_bytes, &app,
                     &prep, nullptr, stream);
}

}  // extern "C"
