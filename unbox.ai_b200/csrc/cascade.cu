// Shared-prefix (cascade) decode attention for radix-shared pages (sm_100a).
//
// The reference's radix cache hands several requests the same physical pages
// for a common prompt prefix (unbox_platform/infer/kvcache.py:97-122, prefix
// match producing shared block tables); paged_decode_attention_ref then reads
// those pages once per request. Here a decode step is split in three:
//   1. the decode kernel attends each request over its private suffix pages
//      (positions past the shared prefix) and also returns the log-sum-exp;
//   2. cascade_prefix_kernel attends every request of a prefix group over the
//      shared pages at once: a CTA loads a chunk of up to 8 shared pages of one
//      KV head into shared memory once, with the q rows of up to 128 (request,
//      query head) pairs of that group, and runs S = Q K^T and O = P V as two
//      chains of 5th-generation tensor-core MMAs (tcgen05.mma, M = 128, fp32
//      accumulators in tensor memory), the softmax in between on one thread per
//      row; it writes unnormalised partial (acc, max, sum) rows per chunk;
//   3. cascade_merge_kernel merges the suffix output with the chunks' partials by
//      log-sum-exp weights (the same combination the split-KV path uses).
// The result equals attention over the whole context (softmax is exactly
// decomposable over disjoint key sets).
#include <type_traits>

#include "ubx_common.cuh"
#include "ubx_internal.h"
#include "ubx_mma.cuh"
#include "ubx_tcgen05.cuh"

namespace ubx {

namespace {

// Shared-memory layout of one prefix CTA (tcgen05 operands, SWIZZLE_NONE
// canonical layout: a tile of R rows x C 16-byte chunks is stored chunk-major,
// [chunk][row][16 B], so 8 consecutive rows of one chunk form a contiguous
// 128-byte core matrix):
//   Q [D/8][128 rows][16 B]  (rows = (member, query head), member-major)
//   K [D/8][128 tokens][16 B], V [D/8][128 tokens][16 B]
//   P [128/8 token chunks][128 rows][16 B] over Q and K once S is complete
//   2 mbarriers, the TMEM base address, the row max / sum of each half [2][128]
constexpr int kTcRows = kCascadeRows;               // M of both MMAs
constexpr int kTcTokens = kCascadeMaxPages * 16;    // N of S, K of O (at most)
constexpr uint32_t kTcCols = 256;                   // TMEM: S (128 columns) + O (head_dim <= 128)
constexpr int kTcThreads = 256;                     // two threads per row: one per column half
constexpr int kTcTailBytes = 64 + 2 * 2 * kTcRows * 4 + (kCascadeMaxPages + kTcRows) * 4;

template <typename T, int D>
__global__ void __launch_bounds__(kTcThreads) cascade_prefix_kernel(const CascadeParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int CH = D / 8;  // 16-byte chunks of a head row
  constexpr int R = kTcRows, TT = kTcTokens, NTH = kTcThreads;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  uint8_t* q_s = smem;
  uint8_t* k_s = q_s + CH * R * 16;
  uint8_t* v_s = k_s + CH * TT * 16;
  uint8_t* p_s = smem;
  uint64_t* bar = reinterpret_cast<uint64_t*>(v_s + CH * TT * 16);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 2);
  float* red_max = reinterpret_cast<float*>(smem + 3 * CH * R * 16 + 64);  // [2][R], 16-byte aligned
  float* red_sum = red_max + 2 * R;                                        // [2][R]
  int32_t* pg_s = reinterpret_cast<int32_t*>(red_sum + 2 * R);             // the chunk's page ids
  int32_t* mem_s = pg_s + kCascadeMaxPages;                                // the item's member sequences
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.y;
  // Launched with programmatic overlap, this CTA may run while the previous
  // kernel drains: it reads only the plan arrays and the shared pages before
  // griddepcontrol.wait (the caller's promise), and q, the workspace and the
  // error word after it. Without the launch attribute the wait returns at once.
  griddep_launch_dependents();
  const int32_t* item = p.work + kCascadeWorkInts * blockIdx.x;
  const int m_off = __ldg(item + 0), n_mem = __ldg(item + 1), pg_off = __ldg(item + 2), n_pg = __ldg(item + 3),
            chunk = __ldg(item + 4);
  const int G = p.num_heads / p.num_kv_heads;
  if (n_pg < 1 || n_pg > kCascadeMaxPages || n_mem < 1 || n_mem * G > R || chunk < 0 || chunk >= p.max_chunks) {
    griddep_wait();
    if (tid == 0) set_error(p.error, kErrBadWork);
    return;
  }
  const int NT = n_pg * 16;  // tokens of this chunk: N of S, K of O (a multiple of 16)
  if (warp == 0) tc::tmem_alloc(tmem_slot, kTcCols);
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  // the item's page ids and member sequences, read once (plan arrays)
  if (tid < n_pg) pg_s[tid] = __ldg(&p.page_list[pg_off + tid]);
  if (tid >= 128 && tid - 128 < n_mem) mem_s[tid - 128] = __ldg(&p.member_list[m_off + tid - 128]);
  __syncthreads();

  // ---- K and V of the chunk's pages (this KV head): 16-byte pieces, 8
  // consecutive lanes = 8 consecutive tokens of one chunk (one core matrix)
  bool bad_page = false;
  for (int v = tid; v < 2 * NT * CH; v += NTH) {
    const int is_v = v >= NT * CH;
    const int u = is_v ? v - NT * CH : v;
    const int t = (u / (8 * CH)) * 8 + (u & 7), c = (u >> 3) % CH;
    uint8_t* dst = (is_v ? v_s : k_s) + (c * TT + t) * 16;
    const int page = pg_s[t >> 4];
    if (page >= 0 && (int64_t)page < p.num_blocks) {
      const uint8_t* src = static_cast<const uint8_t*>(is_v ? p.v_cache : p.k_cache) +
                           ((int64_t)page * p.c_sblk + (int64_t)(t & 15) * p.c_stok + (int64_t)kvh * D) * sizeof(T) +
                           c * 16;
      cp_async_16(dst, src);
    } else {
      if ((t & 15) == 0 && c == 0 && !is_v) bad_page = true;
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  griddep_wait();  // the page copies stay in flight across the wait
  if (bad_page) set_error(p.error, kErrBadPage);
  // ---- Q rows: row r = (member r / G, query head kvh * G + r % G); rows past
  // the members are zero
  for (int v = tid; v < R * CH; v += NTH) {
    const int r = (v / (8 * CH)) * 8 + (v & 7), c = (v >> 3) % CH;
    uint8_t* dst = q_s + (c * R + r) * 16;
    const int mi = r / G;
    const int b = mi < n_mem ? mem_s[mi] : -1;
    if (b >= 0 && b < p.batch) {
      cp_async_16(dst, static_cast<const uint8_t*>(p.q) +
                           ((int64_t)b * p.q_sb + (int64_t)(kvh * G + r % G) * p.q_sh) * sizeof(T) + c * 16);
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_commit_wait_all();
  fence_proxy_async_smem();  // these generic-proxy writes before the MMAs' reads
  tc::fence_before_thread_sync();
  __syncthreads();
  tc::fence_after_thread_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_o = tmem + TT;  // columns [0, 128) and [128, 128 + D)

  // ---- S = Q K^T (M = 128 rows, N = NT tokens, K = D): A and B K-major
  if (tid == 0) {
    const uint32_t idesc = tc::instr_desc_f16(kBf16, R, NT, false, false);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks)
      tc::mma_f16(tmem_s, tc::smem_desc(q_s + ks * 2 * R * 16, R * 16, 128),
                  tc::smem_desc(k_s + ks * 2 * TT * 16, TT * 16, 128), idesc, ks > 0);
    tc::commit(&bar[0]);
  }
  bool ok = mbar_wait_bounded(&bar[0], 0);
  tc::fence_after_thread_sync();

  // ---- softmax: warp w reads TMEM lanes 32 (w % 4) ..; thread = (row, column
  // half h): tokens [64 h, 64 h + 64) of its row
  const int row = (warp & 3) * 32 + lane, h = warp >> 2;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  const int c0 = h * (TT / 2);
  const float cs = p.scale_log2;
  float s[TT / 2];
#pragma unroll
  for (int j = 0; j < TT / 32; ++j) {
    if (c0 + j * 16 < NT) {
      float v16[16];
      tc::ld16(tmem_s + lane_off + c0 + j * 16, v16);
#pragma unroll
      for (int i = 0; i < 16; ++i) s[j * 16 + i] = v16[i];
    }
  }
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < TT / 2; ++j)
    if (c0 + j < NT) mx = fmaxf(mx, s[j]);
  red_max[h * R + row] = mx;
  __syncthreads();
  mx = fmaxf(red_max[row], red_max[R + row]);
  const float mc = mx * cs;
  float l = 0.f;
#pragma unroll
  for (int j8 = 0; j8 < TT / 16; ++j8) {
    if (c0 + j8 * 8 < NT) {
      float pv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        pv[i] = exp2f(fmaf(s[j8 * 8 + i], cs, -mc));
        l += pv[i];
      }
      *reinterpret_cast<uint4*>(p_s + ((c0 / 8 + j8) * R + row) * 16) = Elem<T>::pack(pv);
    }
  }
  red_sum[h * R + row] = l;
  fence_proxy_async_smem();
  tc::fence_before_thread_sync();
  __syncthreads();
  tc::fence_after_thread_sync();

  // ---- O = P V (M = 128 rows, N = D, K = NT tokens): P K-major, V MN-major
  if (tid == 0) {
    const uint32_t idesc = tc::instr_desc_f16(kBf16, R, D, false, true);
    for (int ks = 0; ks < NT / 16; ++ks)
      tc::mma_f16(tmem_o, tc::smem_desc(p_s + ks * 2 * R * 16, R * 16, 128),
                  tc::smem_desc(v_s + ks * 2 * 128, 128, TT * 16), idesc, ks > 0);
    tc::commit(&bar[1]);
  }
  ok = mbar_wait_bounded(&bar[1], 0) && ok;
  tc::fence_after_thread_sync();

  // ---- partial rows of this chunk: unnormalised O and (max in log2 units,
  // sum). Staged through shared memory (rows of D floats + 16 bytes: 8
  // consecutive rows fall in 8 different 16-byte bank groups) over Q, K and V,
  // all consumed, then written row by row with whole warps on each row.
  constexpr int HD = D / 2;
  constexpr int OP = D * 4 + 16;  // staged row pitch (bytes)
  uint8_t* o_s = smem;
  int64_t* slot_s = reinterpret_cast<int64_t*>(red_max);  // [R], over the row max (consumed)
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) {
    float o8[8];
    tc::ld8(tmem_o + lane_off + h * HD + j * 8, o8);
    float4* dst = reinterpret_cast<float4*>(o_s + row * OP + (h * HD + j * 8) * 4);
    dst[0] = make_float4(o8[0], o8[1], o8[2], o8[3]);
    dst[1] = make_float4(o8[4], o8[5], o8[6], o8[7]);
  }
  if (h == 0) {
    const int mi = row / G;
    const int b = mi < n_mem ? mem_s[mi] : -1;
    const bool real = ok && b >= 0 && b < p.batch;
    const int64_t slot = ((int64_t)b * p.num_heads + kvh * G + row % G) * p.max_chunks + chunk;
    slot_s[row] = real ? slot : -1;
    if (real) p.part_ml[slot] = make_float2(mc, red_sum[row] + red_sum[R + row]);
  }
  __syncthreads();
  for (int v = tid; v < R * (D / 4); v += NTH) {
    const int r = v / (D / 4), q4 = v - r * (D / 4);
    const int64_t slot = slot_s[r];
    if (slot >= 0)
      reinterpret_cast<float4*>(p.part_o + slot * D)[q4] = *reinterpret_cast<const float4*>(o_s + r * OP + q4 * 16);
  }
  if (!ok && tid == 0) set_error(p.error, kErrTimeout);
  tc::fence_before_thread_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_thread_sync();
    tc::tmem_dealloc(tmem, kTcCols);
  }
}

// One warp task per (merge item, group of 32 / (D / 8) query heads); lanes are
// (head, 16-byte output chunk). Part 0 is the suffix pass: its normalised
// output row with weight 2^lse (acc = row, max = lse, sum = 1); parts 1.. are
// the prefix chunks. Parts are read kMergeBatch at a time, every load of a
// batch issued before any is used, and folded in with a running max: a merge
// of up to kMergeBatch chunks costs about two memory round trips.
constexpr int kMergeBatch = 8;

template <typename T, int D>
__device__ __forceinline__ void merge_task(const CascadeMergeParams& p, int64_t task, int hgroups, int lane) {
  constexpr int EPC = Elem<T>::kPerChunk;
  constexpr int DCH = D / EPC;   // output chunks per row
  constexpr int HPW = 32 / DCH;  // heads per warp
  const int it = (int)(task / hgroups);
  const int h = (int)(task % hgroups) * HPW + lane / DCH, c = lane % DCH;
  const int b = __ldg(&p.items[2 * it]), nch = __ldg(&p.items[2 * it + 1]);
  if (b < 0 || b >= p.batch || nch < 0 || nch > p.max_chunks) {
    if (lane == 0) set_error(p.error, kErrBadWork);
    return;
  }
  if (lane >= HPW * DCH || h >= p.num_heads) return;  // no warp collectives below
  const int64_t slot0 = ((int64_t)b * p.num_heads + h) * p.max_chunks;
  T* row = static_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + c * EPC;
  const float lse = p.lse[(int64_t)b * p.num_heads + h];  // -inf: empty suffix
  float o[EPC];
  Elem<T>::unpack(*reinterpret_cast<const uint4*>(row), o);
  float M = lse, L = 1.f;
  if (lse == -INFINITY) {
    L = 0.f;
#pragma unroll
    for (int e = 0; e < EPC; ++e) o[e] = 0.f;
  }
  for (int k0 = 0; k0 < nch; k0 += kMergeBatch) {
    float2 ml[kMergeBatch];
    float4 v[kMergeBatch][EPC / 4];
#pragma unroll
    for (int j = 0; j < kMergeBatch; ++j) {
      const bool have = k0 + j < nch;
      const int64_t slot = slot0 + k0 + (have ? j : 0);
      ml[j] = have ? __ldcg(&p.part_ml[slot]) : make_float2(-INFINITY, 0.f);
      const float4* src = reinterpret_cast<const float4*>(p.part_o + slot * D + c * EPC);
#pragma unroll
      for (int e4 = 0; e4 < EPC / 4; ++e4) v[j][e4] = have ? __ldcg(src + e4) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < kMergeBatch; ++j) {
      if (ml[j].x == -INFINITY) continue;  // past the last chunk
      if (ml[j].x > M) {
        const float sc = exp2f(M - ml[j].x);  // M = -inf (empty suffix, first part): 0
        L *= sc;
#pragma unroll
        for (int e = 0; e < EPC; ++e) o[e] *= sc;
        M = ml[j].x;
      }
      const float w = exp2f(ml[j].x - M);
      L = fmaf(ml[j].y, w, L);
#pragma unroll
      for (int e4 = 0; e4 < EPC / 4; ++e4) {
        o[4 * e4 + 0] = fmaf(w, v[j][e4].x, o[4 * e4 + 0]);
        o[4 * e4 + 1] = fmaf(w, v[j][e4].y, o[4 * e4 + 1]);
        o[4 * e4 + 2] = fmaf(w, v[j][e4].z, o[4 * e4 + 2]);
        o[4 * e4 + 3] = fmaf(w, v[j][e4].w, o[4 * e4 + 3]);
      }
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int e = 0; e < EPC; ++e) o[e] *= inv;
  *reinterpret_cast<uint4*>(row) = Elem<T>::pack(o);
}

// One warp per task.
template <typename T, int D>
__global__ void __launch_bounds__(128) cascade_merge_kernel(const CascadeMergeParams p) {
  constexpr int HPW = 32 / (D / Elem<T>::kPerChunk);
  const int lane = threadIdx.x & 31;
  griddep_launch_dependents();
  griddep_wait();  // the suffix and prefix passes have completed
  const int hgroups = (p.num_heads + HPW - 1) / HPW;
  const int64_t t = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t < (int64_t)p.num_items * hgroups) merge_task<T, D>(p, t, hgroups, lane);
}

// Launch with or without programmatic dependent launch (the kernel may start
// while the previous kernel on the stream drains).
template <typename Params>
cudaError_t launch_overlapped(void (*kernel)(const Params), dim3 grid, dim3 block, int smem, cudaStream_t st,
                              bool overlap, const Params& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_prefix_t(int head_dim, const CascadeParams& p, int smem, cudaStream_t st) {
  void (*kernel)(const CascadeParams);
  int slot;
  switch (head_dim) {
    case 64: kernel = cascade_prefix_kernel<T, 64>, slot = 0; break;
    case 112: kernel = cascade_prefix_kernel<T, 112>, slot = 1; break;
    case 128: kernel = cascade_prefix_kernel<T, 128>, slot = 2; break;
    default: return cudaErrorInvalidValue;
  }
  // the shared-memory opt-in is per kernel and per device
  static int attr_done[3][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[slot][dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_done[slot][dev] = 1;
  }
  return launch_overlapped(kernel, dim3(p.num_work, p.num_kv_heads), dim3(kTcThreads), smem, st, p.overlap, p);
}

template <typename T>
cudaError_t launch_merge_t(int head_dim, const CascadeMergeParams& p, cudaStream_t st) {
  const int hpw = 32 / (head_dim / 8);  // heads per warp (16-byte chunks of 16-bit elements)
  const int64_t warps = (int64_t)p.num_items * ((p.num_heads + hpw - 1) / hpw);
  const dim3 blocks((unsigned)((warps + 3) / 4));
  switch (head_dim) {
    case 64: return launch_overlapped(cascade_merge_kernel<T, 64>, blocks, dim3(128), 0, st, p.overlap, p);
    case 112: return launch_overlapped(cascade_merge_kernel<T, 112>, blocks, dim3(128), 0, st, p.overlap, p);
    case 128: return launch_overlapped(cascade_merge_kernel<T, 128>, blocks, dim3(128), 0, st, p.overlap, p);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

// Q, K and V tiles of 128 rows of 16-bit elements, two mbarriers and the TMEM
// address; never below 80 KB, so that at most two CTAs share an SM and their
// tensor memory (2 x 256 columns) never has to wait for a free column.
int cascade_smem_bytes(int head_dim) {
  const int need = 3 * kTcRows * head_dim * 2 + kTcTailBytes;
  return need > kCascadeMinSmem ? need : kCascadeMinSmem;
}

cudaError_t launch_cascade_prefix(int dtype, int head_dim, const CascadeParams& p, cudaStream_t stream) {
  if (p.num_work == 0) return cudaSuccess;
  const int smem = cascade_smem_bytes(head_dim);
  return dtype == 1 ? launch_prefix_t<__nv_bfloat16>(head_dim, p, smem, stream)
                    : launch_prefix_t<__half>(head_dim, p, smem, stream);
}

cudaError_t launch_cascade_merge(int dtype, int head_dim, const CascadeMergeParams& p, cudaStream_t stream) {
  if (p.num_items == 0) return cudaSuccess;
  return dtype == 1 ? launch_merge_t<__nv_bfloat16>(head_dim, p, stream) : launch_merge_t<__half>(head_dim, p, stream);
}

}  // namespace ubx
