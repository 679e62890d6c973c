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

// One thread per VEC-byte piece of a (token, K|V, head) row. Grid-stride.
template <int VEC>
__global__ void __launch_bounds__(256) kv_append_kernel(const uint8_t* __restrict__ k_new,
                                                        const uint8_t* __restrict__ v_new, int64_t n_stok_b,
                                                        int64_t n_sh_b, uint8_t* __restrict__ k_cache,
                                                        uint8_t* __restrict__ v_cache, int64_t c_sblk_b,
                                                        int64_t c_stok_b, int64_t c_sh_b,
                                                        const int64_t* __restrict__ slots, int64_t num_tokens,
                                                        int kvh, int row_bytes, int block_size, int64_t num_blocks,
                                                        int32_t* error_word) {
  using V = typename VecT<VEC>::type;
  const int pieces = row_bytes / VEC;
  const int64_t total = num_tokens * 2 * kvh * pieces;
  const int64_t limit = num_blocks * block_size;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % pieces);
    int64_t rest = i / pieces;
    const int h = (int)(rest % kvh);
    rest /= kvh;
    const int which = (int)(rest & 1);
    const int64_t t = rest >> 1;
    const int64_t slot = __ldg(&slots[t]);
    if (slot < 0) continue;  // padding token
    if (slot >= limit) {
      if (c == 0 && h == 0 && which == 0) set_error(error_word, kErrBadSlot);
      continue;
    }
    const int64_t blk = slot / block_size, off = slot % block_size;
    const uint8_t* src = (which ? v_new : k_new) + t * n_stok_b + h * n_sh_b + (int64_t)c * VEC;
    uint8_t* dst = (which ? v_cache : k_cache) + blk * c_sblk_b + off * c_stok_b + h * c_sh_b + (int64_t)c * VEC;
    *reinterpret_cast<V*>(dst) = *reinterpret_cast<const V*>(src);
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
  const int64_t total = num_tokens * 2 * num_kv_heads * (row_bytes / vec_bytes);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks64 = (total + threads - 1) / threads;
  const int blocks = (int)(blocks64 < 148 * 16 ? blocks64 : 148 * 16);
#define UBX_APPEND(VB)                                                                                          \
  kv_append_kernel<VB><<<blocks, threads, 0, stream>>>(                                                         \
      static_cast<const uint8_t*>(k_new), static_cast<const uint8_t*>(v_new), n_stok_b, n_sh_b,                 \
      static_cast<uint8_t*>(k_cache), static_cast<uint8_t*>(v_cache), c_sblk_b, c_stok_b, c_sh_b, slots,        \
      num_tokens, num_kv_heads, row_bytes, block_size, num_blocks, error_word)
  switch (vec_bytes) {
    case 16: UBX_APPEND(16); break;
    case 8: UBX_APPEND(8); break;
    case 4: UBX_APPEND(4); break;
    case 2: UBX_APPEND(2); break;
    default: return cudaErrorInvalidValue;
  }
#undef UBX_APPEND
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
