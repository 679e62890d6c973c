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
//   * pool -> pool directly, where the destination (a prefill worker pushing)
//     or the source (a decode worker pulling) may be another GPU's memory (peer
//     access or an IPC mapping): the rows cross NVLink as plain loads and
//     stores, with no staging buffer and no host round trip.
// The packed payload has the reference's byte order: (layer, K|V, page, row).
//
// A page unit (one layer, K or V, one page) is page_bytes contiguous bytes in
// both layouts.
#include "ubx_common.cuh"
#include "ubx_internal.h"

namespace ubx {

namespace {

constexpr int kCopyThreads = 256;
constexpr int kUnroll = 4;

// Division by a loop-invariant divisor d (Granlund & Montgomery, "Division by
// invariant integers using multiplication", 1994): with s = ceil(log2 d) and
// m = floor(2^32 (2^s - d) / d) + 1, n / d = (umulhi(n, m) + n) >> s for every
// 32-bit n (the sum is formed in 64 bits).
struct FastDiv {
  uint32_t d, m, s;
};

FastDiv make_fast_div(uint32_t d) {
  uint32_t s = 0;
  while (((uint64_t)1 << s) < d) ++s;
  const uint64_t m = (((uint64_t)1 << 32) * (((uint64_t)1 << s) - d)) / d + 1;
  return FastDiv{d, (uint32_t)m, s};
}

__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv& f) {
  return (uint32_t)(((uint64_t)__umulhi(n, f.m) + n) >> f.s);
}

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

// The copy is one flat array of 16-byte vectors in payload order (unit u =
// (layer, K|V, page) holds vectors [u * vpu, (u + 1) * vpu)); every thread takes
// the same share of it, grid-stride, so no CTA is left with an extra page at the
// end. Four vectors per thread are in flight.
template <bool CHECKSUM>
__global__ void __launch_bounds__(kCopyThreads) kv_pages_copy_kernel(const PageSide src, const PageSide dst,
                                                                    const FastDiv vpu_div, const FastDiv np_div,
                                                                    uint32_t total, unsigned long long* checksum,
                                                                    int32_t* error) {
  // 32-bit index math: the host keeps one call's vectors below 2^31
  const uint32_t vpu = vpu_div.d;
  const uint32_t np = np_div.d;
  const uint32_t stride = gridDim.x * kCopyThreads;
  uint64_t sum = 0;
  for (uint32_t v0 = blockIdx.x * kCopyThreads + threadIdx.x; v0 < total; v0 += stride * kUnroll) {
    uint4 r[kUnroll];
    uint4* d[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const uint32_t v = v0 + k * stride;
      d[k] = nullptr;
      if (v < total) {
        const uint32_t u = fast_div(v, vpu_div), off = v - u * vpu;
        const uint32_t rest = fast_div(u, np_div);
        const int i = (int)(u - rest * np);
        const int c = (int)(rest & 1u);
        const int l = (int)(rest >> 1);
        bool ok = true;
        const uint4* s = reinterpret_cast<const uint4*>(unit_addr(src, l, c, i, ok));
        uint4* t = reinterpret_cast<uint4*>(const_cast<uint8_t*>(unit_addr(dst, l, c, i, ok)));
        if (ok) {
          r[k] = __ldcs(s + off);  // streamed once: evict first
          d[k] = t + off;
        } else if (off == 0) {
          set_error(error, kErrBadPage);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      if (d[k]) {
        __stcs(d[k], r[k]);
        if constexpr (CHECKSUM) sum += vec_checksum(r[k], 4 * (uint64_t)(v0 + (uint32_t)k * stride));
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

// Local copies go through the TMA engine: a persistent CTA takes an equal
// contiguous share of the copy's pieces (a page unit cut into equal pieces of at
// most 16 KB), thread 0 bulk-loads pieces into a ring of shared-memory stages
// and bulk-stores each one as soon as it lands, so one thread keeps up to
// kBulkStages pieces moving and the SMs issue almost no instructions. With the
// checksum, the CTA's threads add up each piece from shared memory meanwhile.
constexpr int kBulkStages = 4;
constexpr uint32_t kMaxPieceBytes = 16384;
constexpr int kBulkThreads = 128;

struct Piece {
  const uint8_t* src;
  uint8_t* dst;
  uint32_t bytes;
  uint64_t word0;  // payload index of the piece's first 32-bit word
  bool ok;
};

__device__ __forceinline__ Piece piece_at(const PageSide& src, const PageSide& dst, uint32_t q, uint32_t ppu,
                                          uint32_t piece_bytes, uint32_t num_pages, uint64_t page_bytes) {
  const uint32_t u = q / ppu, part = q - u * ppu;
  const uint32_t rest = u / num_pages;
  const int i = (int)(u - rest * num_pages), c = (int)(rest & 1u), l = (int)(rest >> 1);
  Piece pc;
  pc.ok = true;
  const uint64_t off = (uint64_t)part * piece_bytes;
  pc.src = unit_addr(src, l, c, i, pc.ok) + off;
  pc.dst = const_cast<uint8_t*>(unit_addr(dst, l, c, i, pc.ok)) + off;
  pc.bytes = (uint32_t)(page_bytes - off < piece_bytes ? page_bytes - off : piece_bytes);
  pc.word0 = ((uint64_t)u * page_bytes + off) / 4;
  return pc;
}

template <bool CHECKSUM>
__global__ void __launch_bounds__(kBulkThreads) kv_pages_bulk_kernel(const PageSide src, const PageSide dst,
                                                                    uint32_t num_pages, uint64_t page_bytes,
                                                                    uint32_t ppu, uint32_t piece_bytes,
                                                                    uint32_t total_pieces,
                                                                    unsigned long long* checksum, int32_t* error) {
  extern __shared__ __align__(128) uint8_t ring[];  // kBulkStages * piece_bytes
  __shared__ uint64_t full[kBulkStages];
  const int tid = threadIdx.x;
  const uint32_t q0 = (uint32_t)((uint64_t)total_pieces * blockIdx.x / gridDim.x);
  const uint32_t q1 = (uint32_t)((uint64_t)total_pieces * (blockIdx.x + 1) / gridDim.x);
  const int n = (int)(q1 - q0);
  if (tid == 0) {
    for (int st = 0; st < kBulkStages; ++st) mbar_init(&full[st], 1);
    fence_mbar_init();
  }
  __syncthreads();

  int issued = 0;  // pieces whose load thread 0 has issued
  auto issue = [&](int k) {
    const Piece pc = piece_at(src, dst, q0 + k, ppu, piece_bytes, num_pages, page_bytes);
    uint64_t* bar = &full[k % kBulkStages];
    if (pc.ok) {
      mbar_arrive_expect_tx(bar, pc.bytes);
      bulk_copy_g2s(ring + (k % kBulkStages) * piece_bytes, pc.src, pc.bytes, bar);
    } else {
      set_error(error, kErrBadPage);
      mbar_arrive(bar);  // the stage completes empty; nothing is stored
    }
    issued = k + 1;
  };
  if (tid == 0)
    for (int k = 0; k < n && k < kBulkStages; ++k) issue(k);

  uint64_t sum = 0;
  int k = 0;
  if (CHECKSUM || tid == 0) {
    for (; k < n; ++k) {
      const int st = k % kBulkStages;
      const bool landed = mbar_wait_bounded(&full[st], (uint32_t)(k / kBulkStages) & 1u);
      bool stop;
      if constexpr (CHECKSUM) {
        stop = __syncthreads_or(!landed);
      } else {
        stop = !landed;
      }
      if (stop) {
        if (tid == 0) set_error(error, kErrTimeout);
        break;
      }
      const Piece pc = piece_at(src, dst, q0 + k, ppu, piece_bytes, num_pages, page_bytes);
      const uint8_t* stage = ring + st * piece_bytes;
      if (tid == 0) {
        if (pc.ok) {
          fence_proxy_async_smem();
          bulk_copy_s2g(pc.dst, stage, pc.bytes);
        }
        bulk_commit_group();  // one group per piece, empty for a skipped one
      }
      if constexpr (CHECKSUM) {
        if (pc.ok)
          for (uint32_t v = tid; v < pc.bytes / 16; v += kBulkThreads)
            sum += vec_checksum(reinterpret_cast<const uint4*>(stage)[v], pc.word0 + 4 * (uint64_t)v);
        __syncthreads();  // stage st is read by every thread before it is refilled
      }
      // refill the previous piece's stage once its store has read it
      if (tid == 0 && k >= 1 && k - 1 + kBulkStages < n) {
        bulk_wait_group_read<1>();
        issue(k - 1 + kBulkStages);
      }
    }
  }
  if (tid == 0) {
    // after a timeout: let the loads still in flight land (bounded) before the CTA exits
    for (int j = k; j < issued; ++j) mbar_wait_bounded(&full[j % kBulkStages], (uint32_t)(j / kBulkStages) & 1u);
    bulk_wait_group<0>();  // the stores are complete before the CTA's shared memory goes away
  }
  if constexpr (CHECKSUM) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((tid & 31) == 0 && sum) atomicAdd(checksum, (unsigned long long)sum);
  }
}

}  // namespace

cudaError_t launch_kv_pages_copy(const KvCopyParams& p, cudaStream_t stream) {
  const int64_t vecs = (int64_t)p.num_layers * 2 * p.num_pages * (p.page_bytes / 16);
  if (vecs == 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // 256-thread CTAs, 8 per SM (a full SM); fewer when the copy is small
  const int64_t want = (int64_t)sms * 8;
  const int64_t need = (vecs + kCopyThreads * kUnroll - 1) / (kCopyThreads * kUnroll);
  const int grid = (int)(need < want ? need : want);
  const PageSide src{const_cast<uint8_t*>(static_cast<const uint8_t*>(p.src)), p.src_s_layer, p.src_s_kv,
                     p.src_s_block, p.src_pages, p.src_num_blocks};
  const PageSide dst{static_cast<uint8_t*>(p.dst), p.dst_s_layer, p.dst_s_kv, p.dst_s_block, p.dst_pages,
                     p.dst_num_blocks};
  if (!p.cross_gpu) {
    // TMA bulk path: pieces of equal size (a multiple of 16 bytes), at most 16 KB
    const uint32_t ppu = (uint32_t)((p.page_bytes + kMaxPieceBytes - 1) / kMaxPieceBytes);
    const uint32_t piece = (uint32_t)(((p.page_bytes + ppu - 1) / ppu + 15) / 16 * 16);
    const uint32_t pieces = (uint32_t)((int64_t)p.num_layers * 2 * p.num_pages) * ppu;
    const int smem = kBulkStages * (int)piece;
    static int attr_done[64] = {0};
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
      cudaFuncSetAttribute(kv_pages_bulk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBulkStages * 16384);
      cudaFuncSetAttribute(kv_pages_bulk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kBulkStages * 16384);
      attr_done[dev] = 1;
    }
    // three CTAs per SM (3 x 64 KB of stages), never more CTAs than pieces
    const int64_t want_b = (int64_t)sms * 3;
    const int grid_b = (int)(pieces < want_b ? pieces : want_b);
    if (p.checksum)
      kv_pages_bulk_kernel<true><<<grid_b, kBulkThreads, smem, stream>>>(
          src, dst, (uint32_t)p.num_pages, (uint64_t)p.page_bytes, ppu, piece, pieces, p.checksum, p.error);
    else
      kv_pages_bulk_kernel<false><<<grid_b, kBulkThreads, smem, stream>>>(
          src, dst, (uint32_t)p.num_pages, (uint64_t)p.page_bytes, ppu, piece, pieces, nullptr, p.error);
    return cudaGetLastError();
  }
  // a side in another GPU's memory: plain 16-byte loads and stores over NVLink
  const FastDiv vpu_div = make_fast_div((uint32_t)(p.page_bytes / 16));
  const FastDiv np_div = make_fast_div((uint32_t)p.num_pages);
  if (p.checksum)
    kv_pages_copy_kernel<true><<<grid, kCopyThreads, 0, stream>>>(src, dst, vpu_div, np_div, (uint32_t)vecs,
                                                                  p.checksum, p.error);
  else
    kv_pages_copy_kernel<false><<<grid, kCopyThreads, 0, stream>>>(src, dst, vpu_div, np_div, (uint32_t)vecs,
                                                                   nullptr, p.error);
  return cudaGetLastError();
}

}  // namespace ubx
