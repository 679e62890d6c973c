// Shared-prefix (cascade) decode attention for radix-shared pages (sm_100a).
//
// The reference's radix cache hands several requests the same physical pages
// for a common prompt prefix (unbox_platform/infer/kvcache.py:97-122, prefix
// match producing shared block tables); paged_decode_attention_ref then reads
// those pages once per request. Here a decode step is split in three:
//   1. the decode kernel attends each request over its private suffix pages
//      (positions past the shared prefix) and also returns the log-sum-exp;
//   2. the shared-prefix pass attends every request of a prefix group over the
//      shared pages at once: a work item is a run of up to 64 shared pages of
//      one KV head and up to 128 (request, query head) rows of that group,
//      taken 8 pages at a time through shared memory with S = Q K^T and
//      O += P V on the 5th-generation tensor cores (tcgen05.mma, M = 128, fp32
//      accumulators in tensor memory) and an online softmax in between, one
//      thread per row (ubx_cascade_prefix.cuh); it writes one unnormalised
//      partial (acc, max, sum) row per run. It runs here as its own kernel
//      (cascade_prefix_kernel, one item per CTA) or inside the suffix pass's
//      launch (cascade_fused_kernel, paged_decode.cu);
//   3. cascade_merge_kernel merges the suffix output with the runs' partials by
//      log-sum-exp weights (the same combination the split-KV path uses).
// The result equals attention over the whole context (softmax is exactly
// decomposable over disjoint key sets).
#include <type_traits>

#include "ubx_cascade_prefix.cuh"
#include "ubx_common.cuh"
#include "ubx_internal.h"
#include "ubx_mma.cuh"
#include "ubx_tcgen05.cuh"

namespace ubx {

namespace {

// One work item per CTA (blockIdx.x: the item, blockIdx.y: the KV head).
template <typename T, int D>
__global__ void __launch_bounds__(kTcThreads) cascade_prefix_kernel(const __grid_constant__ CascadeParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const PrefixSmem sm = carve_prefix_smem<D>(smem);
  const int tid = threadIdx.x;
  // Launched with programmatic overlap, this CTA may run while the previous
  // kernel drains: it reads only the plan arrays and the shared pages before
  // griddepcontrol.wait (the caller's promise), and q, the workspace and the
  // error word after it. Without the launch attribute the wait returns at once.
  griddep_launch_dependents();
  if (tid < 32) tc::tmem_alloc(sm.tmem_slot, kTcCols);
  if (tid == 0) {
    mbar_init(&sm.bar[0], 1);
    mbar_init(&sm.bar[1], 1);
    mbar_init(&sm.bar[2], 1);
    fence_mbar_init();
  }
  tc::fence_before_thread_sync();
  __syncthreads();
  tc::fence_after_thread_sync();
  const uint32_t tmem = *sm.tmem_slot;
  uint32_t parity = 0;
  prefix_item<T, D>(p, blockIdx.x, blockIdx.y, sm, tmem, parity, tid, [] { __syncthreads(); });
  if (tid < 32) tc::tmem_dealloc(tmem, kTcCols);
}

// One warp task per (merge item, group of 32 / (D / 8) query heads); lanes are
// (head, 16-byte output chunk). Part 0 is the suffix pass: its normalised
// output row with weight 2^lse (acc = row, max = lse, sum = 1); parts 1.. are
// the prefix chunks. Parts are read kMergeBatch at a time, every load of a
// batch issued before any is used, and folded in with a running max: a merge
// of up to kMergeBatch chunks costs about two memory round trips.
constexpr int kMergeBatch = 8;

template <typename T, int D>
__device__ __forceinline__ void merge_task(const CascadeMergeParams& p, int64_t task, int hgroups, int b, int nch,
                                           int lane) {
  constexpr int EPC = Elem<T>::kPerChunk;
  constexpr int DCH = D / EPC;   // output chunks per row
  constexpr int HPW = 32 / DCH;  // heads per warp
  const int h = (int)(task % hgroups) * HPW + lane / DCH, c = lane % DCH;
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
  const int hgroups = (p.num_heads + HPW - 1) / HPW;
  const int64_t t = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  const bool has_task = t < (int64_t)p.num_items * hgroups;
  // the merge item is a plan array (not written by the passes): read it while
  // they drain, one memory round trip off the merge
  const int it = has_task ? (int)(t / hgroups) : 0;
  const int b = has_task ? __ldg(&p.items[2 * it]) : 0, nch = has_task ? __ldg(&p.items[2 * it + 1]) : 0;
  griddep_wait();  // the suffix and prefix passes have completed
  if (has_task) merge_task<T, D>(p, t, hgroups, b, nch, lane);
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

// One work item's tiles (Q, K with P over it, V), mbarriers, page ids and
// members; never below 80 KB, so that at most two CTAs share an SM and their
// tensor memory (2 x 256 columns) never has to wait for a free column.
int cascade_smem_bytes(int head_dim) {
  const int need = head_dim == 64 ? prefix_item_smem_bytes<64>()
                   : head_dim == 112 ? prefix_item_smem_bytes<112>() : prefix_item_smem_bytes<128>();
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
