// KV page hand-off between a prefill and a decode worker (sm_100a).
//
// The reference moves a finished prompt's pages as host bytes over ZMQ:
// KVPool.serialize_blocks gathers data[:, :, block_indices] (layers, K|V,
// pages, page rows) to the CPU and KVPool.deserialize_blocks scatters them into
// the decode worker's pool (unbox_platform/infer/kvcache.py:268-277, called at
// worker.py:175-183 and :217-223). Here one kernel copies whole pages between
// any two page layouts on the device:
//   * pool -> packed wire payload (serialize), with the payload checksum fused;
//   * packed payload -> pool pages (deserialize) at the receiver's own page ids;
//   * pool -> pool directly, where the destination may be another GPU's memory
//     (peer access or an IPC mapping): the rows cross NVLink as plain stores,
//     with no staging buffer and no host round trip.
// The packed payload has the reference's byte order: (layer, K|V, page, row).
//
// A page unit (one layer, K or V, one page) is page_bytes contiguous bytes in
// both layouts; CTAs take units in a grid-stride loop and move them as 16-byte
// vectors, four in flight per thread.
#include "ubx_common.cuh"
#include "ubx_internal.h"

namespace ubx {

namespace {

constexpr int kCopyThreads = 256;
constexpr int kUnroll = 4;

struct PageSide {
  uint8_t* base;
  int64_t s_layer, s_kv, s_block;  // byte strides
  const int32_t* pages;            // null: packed wire layout, page i at position i
  int64_t num_blocks;
};

__device__ __forceinline__ const uint8_t* unit_addr(const PageSide& s, int l, int c, int i, bool& ok) {
  int64_t blk = i;
  if (s.pages) {
    blk = __ldg(&s.pages[i]);
    ok = ok && blk >= 0 && blk < s.num_blocks;
  }
  return s.base + l * s.s_layer + c * s.s_kv + blk * s.s_block;
}

// Checksum term of one 16-byte vector whose first 32-bit word has payload index w:
// sum over its four words of word * (2 * index + 1), mod 2^64.
__device__ __forceinline__ uint64_t vec_checksum(const uint4& v, uint64_t w) {
  const uint64_t a = 2 * w + 1;
  return (uint64_t)v.x * a + (uint64_t)v.y * (a + 2) + (uint64_t)v.z * (a + 4) + (uint64_t)v.w * (a + 6);
}

template <bool CHECKSUM>
__global__ void __launch_bounds__(kCopyThreads) kv_pages_copy_kernel(const PageSide src, const PageSide dst,
                                                                    int num_layers, int num_pages,
                                                                    int64_t page_bytes, unsigned long long* checksum,
                                                                    int32_t* error) {
  const int64_t units = (int64_t)num_layers * 2 * num_pages;
  const int64_t vecs = page_bytes / 16;
  uint64_t sum = 0;
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int i = (int)(u % num_pages);
    const int c = (int)((u / num_pages) & 1);
    const int l = (int)(u / (2 * (int64_t)num_pages));
    bool ok = true;
    const uint4* s = reinterpret_cast<const uint4*>(unit_addr(src, l, c, i, ok));
    uint4* d = reinterpret_cast<uint4*>(const_cast<uint8_t*>(unit_addr(dst, l, c, i, ok)));
    if (!ok) {
      if (threadIdx.x == 0) set_error(error, kErrBadPage);
      continue;
    }
    // payload index of this unit's first 32-bit word (packed order = unit order)
    const uint64_t w0 = (uint64_t)u * (uint64_t)(page_bytes / 4);
    for (int64_t v0 = threadIdx.x; v0 < vecs; v0 += kCopyThreads * kUnroll) {
      uint4 r[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t v = v0 + k * kCopyThreads;
        if (v < vecs) r[k] = __ldcs(s + v);  // streamed once: evict first
      }
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) {
        const int64_t v = v0 + k * kCopyThreads;
        if (v < vecs) {
          __stcs(d + v, r[k]);
          if constexpr (CHECKSUM) sum += vec_checksum(r[k], w0 + 4 * (uint64_t)v);
        }
      }
    }
  }
  if constexpr (CHECKSUM) {
    // integer sums are order-independent: the result does not depend on the schedule
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((threadIdx.x & 31) == 0 && sum) atomicAdd(checksum, (unsigned long long)sum);
  }
}

}  // namespace

cudaError_t launch_kv_pages_copy(const KvCopyParams& p, cudaStream_t stream) {
  const int64_t units = (int64_t)p.num_layers * 2 * p.num_pages;
  if (units == 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // 256-thread CTAs, 8 per SM resident at most; never more CTAs than units
  const int64_t want = (int64_t)sms * 8;
  const int grid = (int)(units < want ? units : want);
  const PageSide src{const_cast<uint8_t*>(static_cast<const uint8_t*>(p.src)), p.src_s_layer, p.src_s_kv,
                     p.src_s_block, p.src_pages, p.src_num_blocks};
  const PageSide dst{static_cast<uint8_t*>(p.dst), p.dst_s_layer, p.dst_s_kv, p.dst_s_block, p.dst_pages,
                     p.dst_num_blocks};
  if (p.checksum)
    kv_pages_copy_kernel<true><<<grid, kCopyThreads, 0, stream>>>(src, dst, p.num_layers, p.num_pages, p.page_bytes,
                                                                  p.checksum, p.error);
  else
    kv_pages_copy_kernel<false><<<grid, kCopyThreads, 0, stream>>>(src, dst, p.num_layers, p.num_pages,
                                                                   p.page_bytes, nullptr, p.error);
  return cudaGetLastError();
}

}  // namespace ubx
