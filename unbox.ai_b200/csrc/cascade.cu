// Shared-prefix (cascade) decode attention for radix-shared pages (sm_100a).
//
// The reference's radix cache hands several requests the same physical pages
// for a common prompt prefix (unbox_platform/infer/kvcache.py:97-122, prefix
// match producing shared block tables); paged_decode_attention_ref then reads
// those pages once per request. Here a decode step is split in three:
//   1. the decode kernel attends each request over its private suffix pages
//      (positions past the shared prefix) and also returns the log-sum-exp;
//   2. cascade_prefix_kernel attends every request of a prefix group over the
//      shared pages at once: a CTA loads a chunk of the shared pages of one KV
//      head into shared memory once, and each warp runs a 16-row tensor-core
//      tile of (request, query head) rows of that group over them (mma.sync
//      m16n8k16, full tiles: G query heads x 16/G requests), writing unnormalised
//      partial (acc, max, sum) rows per chunk;
//   3. cascade_merge_kernel merges the suffix output with the chunks' partials by
//      log-sum-exp weights (the same combination the split-KV path uses).
// The result equals attention over the whole context (softmax is exactly
// decomposable over disjoint key sets).
#include "ubx_common.cuh"
#include "ubx_internal.h"
#include "ubx_mma.cuh"

namespace ubx {

namespace {

constexpr unsigned kAll = 0xffffffffu;

template <typename T, int D>
__global__ void __launch_bounds__(kCascadeWarps * 32) cascade_prefix_kernel(const CascadeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int KS = D / 16;  // QK k-steps
  constexpr int NT = D / 8;   // PV n-tiles
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
  if (n_pg < 1 || n_pg > kCascadeMaxPages || n_mem < 1 || n_mem * G > kCascadeWarps * 16 || chunk < 0 ||
      chunk >= p.max_chunks) {
    griddep_wait();
    if (threadIdx.x == 0) set_error(p.error, kErrBadWork);
    return;
  }
  constexpr int kRowBytes = D * (int)sizeof(T);  // one KV head row of one token
  constexpr int kVecPerRow = kRowBytes / 16;
  const int tile = kBlockSize * p.pitch;          // one page of this head, K or V
  uint8_t* k_s = smem;
  uint8_t* v_s = smem + n_pg * tile;

  // ---- load: every thread copies 16-byte pieces of the chunk's K and V rows of
  // this head (cp.async, no register staging); rows of a bad page are zeroed
  const int total = n_pg * 2 * kBlockSize * kVecPerRow;
  bool bad_page = false;
  for (int v = threadIdx.x; v < total; v += kCascadeWarps * 32) {
    const int row = v / kVecPerRow, cv = v - row * kVecPerRow;
    const int i = row / (2 * kBlockSize), r = row % (2 * kBlockSize);
    const bool is_v = r >= kBlockSize;
    const int tok = r & (kBlockSize - 1);
    uint8_t* dst = (is_v ? v_s : k_s) + i * tile + tok * p.pitch + cv * 16;
    const int page = __ldg(&p.page_list[pg_off + i]);
    if (page >= 0 && (int64_t)page < p.num_blocks) {
      const uint8_t* src = static_cast<const uint8_t*>(is_v ? p.v_cache : p.k_cache) +
                           ((int64_t)page * p.c_sblk + (int64_t)tok * p.c_stok + (int64_t)kvh * D) * sizeof(T) +
                           cv * 16;
      cp_async_16(dst, src);
    } else {
      if (tok == 0 && cv == 0 && !is_v) bad_page = true;
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  griddep_wait();  // the page copies stay in flight across the wait
  if (bad_page) set_error(p.error, kErrBadPage);
  cp_async_commit_wait_all();
  __syncthreads();

  // ---- tiles: 16 rows = (request, query head), request-major; G heads x 16/G requests
  const int MT = 16 / G;
  const int n_tiles = (n_mem + MT - 1) / MT;
  const int qr = lane >> 2, qc = lane & 3;
  const float c = p.scale_log2;
  const int rs = p.pitch / (int)sizeof(T);
  const int k_row = (((lane >> 4) & 1) * 8 + (lane & 7)) * rs + ((lane >> 3) & 1) * 8;
  const int v_row = (((lane >> 3) & 1) * 8 + (lane & 7)) * rs + ((lane >> 4) & 1) * 8;
  for (int t = warp; t < n_tiles; t += kCascadeWarps) {
    int bs[2], head[2];
    bool real[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = qr + 8 * h, mi = t * MT + r / G;
      real[h] = mi < n_mem;
      bs[h] = real[h] ? __ldg(&p.member_list[m_off + mi]) : 0;
      real[h] = real[h] && bs[h] >= 0 && bs[h] < p.batch;
      head[h] = kvh * G + r % G;
    }
    uint32_t qa[KS][4];
    {
      const T* q0 = static_cast<const T*>(p.q) + (int64_t)bs[0] * p.q_sb + (int64_t)head[0] * p.q_sh;
      const T* q1 = static_cast<const T*>(p.q) + (int64_t)bs[1] * p.q_sb + (int64_t)head[1] * p.q_sh;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qa[ks][0] = real[0] ? __ldg(reinterpret_cast<const uint32_t*>(q0 + 16 * ks + 2 * qc)) : 0u;
        qa[ks][1] = real[1] ? __ldg(reinterpret_cast<const uint32_t*>(q1 + 16 * ks + 2 * qc)) : 0u;
        qa[ks][2] = real[0] ? __ldg(reinterpret_cast<const uint32_t*>(q0 + 16 * ks + 8 + 2 * qc)) : 0u;
        qa[ks][3] = real[1] ? __ldg(reinterpret_cast<const uint32_t*>(q1 + 16 * ks + 8 + 2 * qc)) : 0u;
      }
    }
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

    // two pages per step: four independent QK accumulation chains, one softmax
    // update over 32 tokens, then PV of both pages
    for (int i = 0; i < n_pg; i += 2) {
      const bool two = i + 1 < n_pg;  // warp-uniform
      const T* kt0 = reinterpret_cast<const T*>(k_s + i * tile);
      const T* kt1 = reinterpret_cast<const T*>(k_s + (two ? i + 1 : i) * tile);
      // S[16 rows x 16 tokens] per page: s[page][n-tile][0..1] row qr, [2..3] row qr + 8
      float sc[2][2][4] = {};
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t r0, r1, r2, r3, u0, u1, u2, u3;
        ldsm_x4(kt0 + k_row + 16 * ks, r0, r1, r2, r3);
        ldsm_x4(kt1 + k_row + 16 * ks, u0, u1, u2, u3);
        mma16816<T>(sc[0][0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], r0, r1);
        mma16816<T>(sc[0][1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], r2, r3);
        mma16816<T>(sc[1][0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], u0, u1);
        mma16816<T>(sc[1][1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], u2, u3);
      }
      if (!two) {  // odd page count: the second page is absent
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[1][nt][e] = -INFINITY;
      }
      float pv[2][2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float mx = -INFINITY;
#pragma unroll
        for (int pg = 0; pg < 2; ++pg)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) mx = fmaxf(mx, fmaxf(sc[pg][nt][2 * h], sc[pg][nt][2 * h + 1]));
        mx = fmaxf(mx, __shfl_xor_sync(kAll, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(kAll, mx, 2));
        const float m_new = fmaxf(m[h], mx);
        if (m_new != m[h]) {  // rescale this row only when its max moved
          const float alpha = exp2f((m[h] - m_new) * c);
          l[h] *= alpha;
#pragma unroll
          for (int n = 0; n < NT; ++n) {
            o[n][2 * h] *= alpha;
            o[n][2 * h + 1] *= alpha;
          }
          m[h] = m_new;
        }
        const float mc = m[h] * c;
#pragma unroll
        for (int pg = 0; pg < 2; ++pg)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            pv[pg][nt][2 * h] = exp2f(fmaf(sc[pg][nt][2 * h], c, -mc));
            pv[pg][nt][2 * h + 1] = exp2f(fmaf(sc[pg][nt][2 * h + 1], c, -mc));
            l[h] += pv[pg][nt][2 * h] + pv[pg][nt][2 * h + 1];
          }
      }
      // P as the A operand of PV (the S accumulator layout is the A layout)
#pragma unroll
      for (int pg = 0; pg < 2; ++pg) {
        if (pg == 1 && !two) break;
        const T* vt = reinterpret_cast<const T*>(v_s + (i + pg) * tile);
        const uint32_t pa0 = Elem<T>::pack2(pv[pg][0][0], pv[pg][0][1]);
        const uint32_t pa1 = Elem<T>::pack2(pv[pg][0][2], pv[pg][0][3]);
        const uint32_t pa2 = Elem<T>::pack2(pv[pg][1][0], pv[pg][1][1]);
        const uint32_t pa3 = Elem<T>::pack2(pv[pg][1][2], pv[pg][1][3]);
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
          uint32_t r0, r1, r2, r3;
          ldsm_x4_trans(vt + v_row + 16 * np, r0, r1, r2, r3);
          mma16816<T>(o[2 * np], pa0, pa1, pa2, pa3, r0, r1);
          mma16816<T>(o[2 * np + 1], pa0, pa1, pa2, pa3, r2, r3);
        }
      }
    }
    // ---- partial rows of this chunk
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float lt = l[h];
      lt += __shfl_xor_sync(kAll, lt, 1);
      lt += __shfl_xor_sync(kAll, lt, 2);
      if (!real[h]) continue;
      const int64_t slot = ((int64_t)bs[h] * p.num_heads + head[h]) * p.max_chunks + chunk;
      float2* dst = reinterpret_cast<float2*>(p.part_o + slot * D + 2 * qc);
#pragma unroll
      for (int n = 0; n < NT; ++n) dst[4 * n] = make_float2(o[n][2 * h], o[n][2 * h + 1]);
      if (qc == 0) p.part_ml[slot] = make_float2(m[h] * c, lt);
    }
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
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kCascadeMaxSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_done[slot][dev] = 1;
  }
  return launch_overlapped(kernel, dim3(p.num_work, p.num_kv_heads), dim3(kCascadeWarps * 32), smem, st, p.overlap,
                           p);
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

int cascade_smem_bytes(int head_dim, int elem_bytes, int num_pages) {
  return num_pages * 2 * kBlockSize * tile_row_pitch(head_dim * elem_bytes);
}

cudaError_t launch_cascade_prefix(int dtype, int head_dim, const CascadeParams& p, cudaStream_t stream) {
  if (p.num_work == 0) return cudaSuccess;
  const int smem = cascade_smem_bytes(head_dim, 2, kCascadeMaxPages);
  return dtype == 1 ? launch_prefix_t<__nv_bfloat16>(head_dim, p, smem, stream)
                    : launch_prefix_t<__half>(head_dim, p, smem, stream);
}

cudaError_t launch_cascade_merge(int dtype, int head_dim, const CascadeMergeParams& p, cudaStream_t stream) {
  if (p.num_items == 0) return cudaSuccess;
  return dtype == 1 ? launch_merge_t<__nv_bfloat16>(head_dim, p, stream) : launch_merge_t<__half>(head_dim, p, stream);
}

}  // namespace ubx
