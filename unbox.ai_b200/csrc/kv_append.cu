// KV append and slot mapping for one decode step (sm_100a).
//
// kv_append replaces the engine's per-sequence write loop
// (unbox_platform/infer/engine.py:213-215 -> PagedKVCache.write_kv,
// kvcache.py:330-340 -> KVPool.write_kv, kvcache.py:253-262) with one launch
// that scatters every new K and V row to its page slot. The rows are copied as
// raw bytes (bit-exact), 16 bytes per thread when every row and stride allows it.
#include "ubx_common.cuh"
#include "ubx_internal.h"

namespace ubx {

namespace {

template <int VEC>
struct VecT;
template <>
struct VecT<16> { using type = uint4; };
template <>
struct VecT<8> { using type = uint2; };
template <>
struct VecT<4> { using type = uint32_t; };
template <>
struct VecT<2> { using type = uint16_t; };

// Copy one (token, K|V) row of kvh head rows (row_bytes each) with the 32
// lanes of a warp, VEC bytes per access, 32-bit offsets inside the row. FLAT:
// the heads are contiguous in both the new rows and the pool, so the row is one
// contiguous span on each side.
template <int VEC, bool FLAT>
__device__ __forceinline__ void copy_row(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t n_sh_b,
                                         int64_t c_sh_b, int kvh, int row_bytes, int lane) {
  using V = typename VecT<VEC>::type;
  const int pieces = row_bytes / VEC;
  if constexpr (FLAT) {
    // four loads in flight per lane before their stores
    const int per_tok = kvh * pieces;
    for (int base = lane; base < per_tok; base += 4 * 32) {
      V r[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (base + 32 * k < per_tok) r[k] = *reinterpret_cast<const V*>(src + (base + 32 * k) * VEC);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (base + 32 * k < per_tok) *reinterpret_cast<V*>(dst + (base + 32 * k) * VEC) = r[k];
    }
  } else {
    for (int h = 0; h < kvh; ++h)
      for (int c = lane; c < pieces; c += 32)
        *reinterpret_cast<V*>(dst + h * c_sh_b + c * VEC) = *reinterpret_cast<const V*>(src + h * n_sh_b + c * VEC);
  }
}

// One warp per (token, K|V) row, grid-stride over rows; the slot is read once per row.
template <int VEC, bool FLAT>
__global__ void __launch_bounds__(256) kv_append_kernel(const uint8_t* __restrict__ k_new,
                                                        const uint8_t* __restrict__ v_new, int64_t n_stok_b,
                                                        int64_t n_sh_b, uint8_t* __restrict__ k_cache,
                                                        uint8_t* __restrict__ v_cache, int64_t c_sblk_b,
                                                        int64_t c_stok_b, int64_t c_sh_b,
                                                        const int64_t* __restrict__ slots, int64_t num_tokens,
                                                        int kvh, int row_bytes, int block_size, int64_t num_blocks,
                                                        int32_t* error_word) {
  const int64_t limit = num_blocks * block_size;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < 2 * num_tokens; r += nwarps) {
    const int64_t t = r >> 1;
    const int which = (int)(r & 1);
    const int64_t slot = __ldg(&slots[t]);
    if (slot < 0) continue;  // padding token
    if (slot >= limit) {
      if (lane == 0 && which == 0) set_error(error_word, kErrBadSlot);
      continue;
    }
    const int64_t blk = slot / block_size;
    const int off = (int)(slot - blk * block_size);
    copy_row<VEC, FLAT>((which ? v_new : k_new) + t * n_stok_b,
                        (which ? v_cache : k_cache) + blk * c_sblk_b + (int64_t)off * c_stok_b, n_sh_b, c_sh_b, kvh,
                        row_bytes, lane);
  }
}

// Prefill chunk: tokens t = 0 .. T-1 of one sequence at positions start + t;
// the slot is computed here from the sequence's block-table row (the same
// rule as slot_mapping_kernel: past the row or a negative page = no slot) and
// optionally stored to slots_out.
template <int VEC, bool FLAT>
__global__ void __launch_bounds__(256) prefill_append_kernel(const uint8_t* __restrict__ k_new,
                                                             const uint8_t* __restrict__ v_new, int64_t n_stok_b,
                                                             int64_t n_sh_b, uint8_t* __restrict__ k_cache,
                                                             uint8_t* __restrict__ v_cache, int64_t c_sblk_b,
                                                             int64_t c_stok_b, int64_t c_sh_b,
                                                             const int32_t* __restrict__ bt_row, int max_blocks,
                                                             int64_t start_pos, int64_t num_tokens, int kvh,
                                                             int row_bytes, int block_size, int64_t num_blocks,
                                                             int64_t* __restrict__ slots_out, int32_t* error_word) {
  const int64_t limit = num_blocks * block_size;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  // launched with programmatic overlap: the next kernel may launch now, and
  // nothing is read or written before the previous kernel has completed
  griddep_launch_dependents();
  griddep_wait();
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < 2 * num_tokens; r += nwarps) {
    const int64_t t = r >> 1;
    const int which = (int)(r & 1);
    const int64_t pos = start_pos + t;
    int64_t slot = -1;
    if (pos >= 0 && pos / block_size < max_blocks) {
      const int page = __ldg(&bt_row[pos / block_size]);
      if (page >= 0) slot = (int64_t)page * block_size + pos % block_size;
    }
    if (slots_out != nullptr && which == 0 && lane == 0) slots_out[t] = slot;
    if (slot < 0) continue;
    if (slot >= limit) {
      if (lane == 0 && which == 0) set_error(error_word, kErrBadSlot);
      continue;
    }
    const int64_t blk = slot / block_size;
    const int off = (int)(slot - blk * block_size);
    copy_row<VEC, FLAT>((which ? v_new : k_new) + t * n_stok_b,
                        (which ? v_cache : k_cache) + blk * c_sblk_b + (int64_t)off * c_stok_b, n_sh_b, c_sh_b, kvh,
                        row_bytes, lane);
  }
}

__global__ void slot_mapping_kernel(const int32_t* __restrict__ block_table, int64_t bt_s_row,
                                    const int32_t* __restrict__ positions, int64_t* __restrict__ slots, int batch,
                                    int max_blocks, int block_size) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int pos = positions[b];
  int64_t slot = -1;
  if (pos >= 0 && pos / block_size < max_blocks) {
    const int page = block_table[(int64_t)b * bt_s_row + pos / block_size];
    if (page >= 0) slot = (int64_t)page * block_size + pos % block_size;
  }
  slots[b] = slot;
}

}  // namespace

cudaError_t launch_kv_append(const void* k_new, const void* v_new, int64_t n_stok_b, int64_t n_sh_b, void* k_cache,
                             void* v_cache, int64_t c_sblk_b, int64_t c_stok_b, int64_t c_sh_b,
                             const int64_t* slots, int64_t num_tokens, int num_kv_heads, int row_bytes,
                             int block_size, int64_t num_blocks, int vec_bytes, int32_t* error_word,
                             cudaStream_t stream) {
  const int64_t rows = num_tokens * 2;  // one warp per (token, K|V) row
  if (rows == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks64 = (rows + 7) / 8;
  const int blocks = (int)(blocks64 < 148 * 8 ? blocks64 : 148 * 8);
  const bool flat = n_sh_b == row_bytes && c_sh_b == row_bytes;
#define UBX_APPEND(VB, FL)                                                                                      \
  kv_append_kernel<VB, FL><<<blocks, threads, 0, stream>>>(                                                     \
      static_cast<const uint8_t*>(k_new), static_cast<const uint8_t*>(v_new), n_stok_b, n_sh_b,                 \
      static_cast<uint8_t*>(k_cache), static_cast<uint8_t*>(v_cache), c_sblk_b, c_stok_b, c_sh_b, slots,        \
      num_tokens, num_kv_heads, row_bytes, block_size, num_blocks, error_word)
  switch (vec_bytes) {
    case 16: if (flat) UBX_APPEND(16, true); else UBX_APPEND(16, false); break;
    case 8: if (flat) UBX_APPEND(8, true); else UBX_APPEND(8, false); break;
    case 4: if (flat) UBX_APPEND(4, true); else UBX_APPEND(4, false); break;
    case 2: if (flat) UBX_APPEND(2, true); else UBX_APPEND(2, false); break;
    default: return cudaErrorInvalidValue;
  }
#undef UBX_APPEND
  return cudaGetLastError();
}

cudaError_t launch_prefill_append(const void* k_new, const void* v_new, int64_t n_stok_b, int64_t n_sh_b,
                                  void* k_cache, void* v_cache, int64_t c_sblk_b, int64_t c_stok_b, int64_t c_sh_b,
                                  const int32_t* bt_row, int max_blocks, int64_t start_pos, int64_t num_tokens,
                                  int num_kv_heads, int row_bytes, int block_size, int64_t num_blocks, int vec_bytes,
                                  int64_t* slots_out, int32_t* error_word, bool overlap, cudaStream_t stream) {
  const int64_t rows = num_tokens * 2;
  if (rows == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks64 = (rows + 7) / 8;
  const int blocks = (int)(blocks64 < 148 * 8 ? blocks64 : 148 * 8);
  const bool flat = n_sh_b == row_bytes && c_sh_b == row_bytes;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap ? 1 : 0;
  cudaError_t e = cudaSuccess;
#define UBX_PREFILL(VB, FL)                                                                                     \
  e = cudaLaunchKernelEx(&cfg, prefill_append_kernel<VB, FL>, static_cast<const uint8_t*>(k_new),               \
                         static_cast<const uint8_t*>(v_new), n_stok_b, n_sh_b, static_cast<uint8_t*>(k_cache),   \
                         static_cast<uint8_t*>(v_cache), c_sblk_b, c_stok_b, c_sh_b, bt_row, max_blocks,         \
                         start_pos, num_tokens, num_kv_heads, row_bytes, block_size, num_blocks, slots_out,       \
                         error_word)
  switch (vec_bytes) {
    case 16: if (flat) UBX_PREFILL(16, true); else UBX_PREFILL(16, false); break;
    case 8: if (flat) UBX_PREFILL(8, true); else UBX_PREFILL(8, false); break;
    case 4: if (flat) UBX_PREFILL(4, true); else UBX_PREFILL(4, false); break;
    case 2: if (flat) UBX_PREFILL(2, true); else UBX_PREFILL(2, false); break;
    default: return cudaErrorInvalidValue;
  }
#undef UBX_PREFILL
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_slot_mapping(const int32_t* block_table, int64_t bt_s_row, const int32_t* positions,
                                int64_t* slot_mapping, int batch, int max_blocks, int block_size,
                                cudaStream_t stream) {
  if (batch == 0) return cudaSuccess;
  slot_mapping_kernel<<<(batch + 127) / 128, 128, 0, stream>>>(block_table, bt_s_row, positions, slot_mapping,
                                                                batch, max_blocks, block_size);
  return cudaGetLastError();
}

}  // namespace ubx
