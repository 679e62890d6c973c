// Paged GQA decode attention for sm_100a.
//
// Semantics follow paged_decode_attention_ref
// (unbox_platform/infer/kernels/paged_decode_attention.py:157-191): for every
// sequence b and query head h, softmax(scale * q . K) V over the first
// context_lens[b] positions, position j read from page block_table[b, j / 16],
// slot j % 16, KV head h / (H / KVH).
//
// Structure (one CTA per SM, persistent):
//   * A page of the pool holds 16 tokens x KVH heads x D elements, contiguous
//     (the KVPool layout, kvcache.py:248-251). One 4-D TMA box
//     (D, 16 tokens, HG heads, 1 page) moves the K tile of a head group and one
//     more the V tile; the box is laid out [head][token][d] in shared memory so
//     every (token, head) row is D elements at a D*sizeof(T) pitch.
//   * Warp NCW is the producer: it walks the CTA's pages, reads the block table
//     32 entries at a time and issues the two TMA loads per page into a ring of
//     `stages` buffers guarded by full/empty mbarriers.
//   * Consumer warp w owns KV head w / WPK of the head group and GW (<= 2) of
//     its query heads, so a K/V row is read from shared memory once for the GQA
//     group. QK: two lanes per token, each holding half of q in registers.
//     Online softmax in the exp2 domain (scale * log2 e folded into q) with
//     warp-shuffle max. PV: lane = (16-byte chunk of D, token group).
//   * Work split: the balanced schedule gives every CTA the same number of
//     pages of the flattened (sequence, page) list, so a CTA may cover the tail
//     of one sequence, whole sequences and the head of another. A sequence
//     split over several CTAs leaves partial (acc, max, sum) triples in the
//     workspace; the warp that finishes a sequence's last part (an atomic
//     counter, no waiting) merges them with log-sum-exp weights. The split
//     schedule instead gives each CTA a fixed chunk of one sequence and a
//     separate combine kernel merges the chunks.
//
// No waits without bounds: every mbarrier wait gives up after ~2^31 clocks,
// records UBX_DEVERR_TIMEOUT and unwinds; the producer then waits (bounded) for
// its own loads in flight before the CTA exits.
#include "ubx_common.cuh"
#include "ubx_internal.h"

namespace ubx {

namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ int pages_of(const DecodeParams& p, int b, bool report) {
  const int ctx = __ldg(&p.context_lens[b]);
  if (ctx < 0) {
    if (report) set_error(p.error, kErrNegCtx);
    return 0;
  }
  int n = (ctx + kBlockSize - 1) / kBlockSize;
  if (n > p.max_blocks) {
    if (report) set_error(p.error, kErrCtxTooLong);
    n = p.max_blocks;
  }
  return n;
}

__device__ __forceinline__ int warp_inclusive_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(kFull, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// prefix[b] = pages of sequences 0..b-1, prefix[B] = total. Whole CTA.
__device__ void build_page_prefix(const DecodeParams& p, int32_t* prefix, int32_t* warp_tot) {
  const int B = p.batch;
  const int nt = blockDim.x;
  const int per = (B + nt - 1) / nt;
  const int b0 = min(B, (int)threadIdx.x * per);
  const int b1 = min(B, b0 + per);
  const bool report = blockIdx.x == 0 && blockIdx.y == 0;
  int local = 0;
  for (int b = b0; b < b1; ++b) local += pages_of(p, b, report);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = nt >> 5;
  const int incl = warp_inclusive_scan(local, lane);
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = lane < nwarps ? warp_tot[lane] : 0;
    v = warp_inclusive_scan(v, lane);
    warp_tot[lane] = v;
  }
  __syncthreads();
  int run = incl - local + (warp > 0 ? warp_tot[warp - 1] : 0);
  for (int b = b0; b < b1; ++b) {
    prefix[b] = run;
    run += pages_of(p, b, false);
  }
  if (threadIdx.x == nt - 1) prefix[B] = run;
  __syncthreads();
}

template <typename T, int D>
__device__ __forceinline__ void write_zero_row(const DecodeParams& p, int b, int head_begin, int head_end, int tid,
                                               int nthreads) {
  constexpr int EPC = Elem<T>::kPerChunk;
  constexpr int DCH = D / EPC;
  const int n = (head_end - head_begin) * DCH;
  for (int i = tid; i < n; i += nthreads) {
    const int h = head_begin + i / DCH, c = i % DCH;
    T* o = reinterpret_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + c * EPC;
    *reinterpret_cast<uint4*>(o) = make_uint4(0, 0, 0, 0);
  }
}

// Merge `nparts` partial triples of one (sequence, query head) and write the
// normalised output row. slot_of(i) gives the workspace slot of part i.
template <typename T, int D, typename SlotFn>
__device__ __forceinline__ void merge_parts(const DecodeParams& p, int b, int h, int nparts, SlotFn slot_of,
                                            int lane) {
  constexpr int EPC = Elem<T>::kPerChunk;
  constexpr int DCH = D / EPC;
  float M = -INFINITY;
  for (int i = lane; i < nparts; i += 32) M = fmaxf(M, __ldcg(&p.part_ml[(int64_t)slot_of(i) * p.num_heads + h]).x);
  M = warp_max(M);
  float L = 0.f;
  for (int i = lane; i < nparts; i += 32) {
    const float2 ml = __ldcg(&p.part_ml[(int64_t)slot_of(i) * p.num_heads + h]);
    L += ml.y * exp2f(ml.x - M);
  }
  L = warp_sum(L);
  if (lane < DCH) {
    float o[EPC];
#pragma unroll
    for (int e = 0; e < EPC; ++e) o[e] = 0.f;
    for (int i = 0; i < nparts; ++i) {
      const int64_t slot = slot_of(i);
      const float w = exp2f(__ldcg(&p.part_ml[slot * p.num_heads + h]).x - M);
      const float4* src = reinterpret_cast<const float4*>(p.part_o + (slot * p.num_heads + h) * D + lane * EPC);
#pragma unroll
      for (int e4 = 0; e4 < EPC / 4; ++e4) {
        const float4 v = __ldcg(src + e4);
        o[4 * e4 + 0] = fmaf(w, v.x, o[4 * e4 + 0]);
        o[4 * e4 + 1] = fmaf(w, v.y, o[4 * e4 + 1]);
        o[4 * e4 + 2] = fmaf(w, v.z, o[4 * e4 + 2]);
        o[4 * e4 + 3] = fmaf(w, v.w, o[4 * e4 + 3]);
      }
    }
    const float inv = 1.f / L;
#pragma unroll
    for (int e = 0; e < EPC; ++e) o[e] *= inv;
    T* dst = reinterpret_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + lane * EPC;
    *reinterpret_cast<uint4*>(dst) = Elem<T>::pack(o);
  }
}

// One page of one KV head for the GW query heads of this warp.
//   kt, vt: [16 tokens][D] tiles of this warp's KV head in shared memory
//   pw:     this warp's probability buffer [GW][16] (rotated per token group)
template <typename T, int D, int GW, bool MASKED>
__device__ __forceinline__ void page_update(const T* __restrict__ kt, const T* __restrict__ vt, int valid,
                                            const float (&qv)[GW][D / 2], float (&m)[GW], float (&l)[GW],
                                            float (&acc)[GW][Elem<T>::kPerChunk], float* pw, int lane) {
  constexpr int EPC = Elem<T>::kPerChunk;
  constexpr int DCH = D / EPC;       // 16-byte chunks per row
  constexpr int CPL = DCH / 2;       // QK: chunks per lane (two lanes per token)
  constexpr int NG = 32 / DCH;       // PV: token groups
  constexpr int TPG = kBlockSize / NG;
  const int t = lane >> 1, half = lane & 1;

  // ---- scores: lane pair (2t, 2t+1) covers token t, each lane half of D
  const uint4* krow = reinterpret_cast<const uint4*>(kt) + t * DCH + half * CPL;
  float sa[GW], sb[GW];
#pragma unroll
  for (int g = 0; g < GW; ++g) sa[g] = sb[g] = 0.f;
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    float kf[EPC];
    Elem<T>::unpack(krow[c], kf);
#pragma unroll
    for (int e = 0; e < EPC; ++e) {
#pragma unroll
      for (int g = 0; g < GW; ++g) {
        if (c & 1)
          sb[g] = fmaf(qv[g][c * EPC + e], kf[e], sb[g]);
        else
          sa[g] = fmaf(qv[g][c * EPC + e], kf[e], sa[g]);
      }
    }
  }
  float alpha[GW];
  bool rescale = false;
#pragma unroll
  for (int g = 0; g < GW; ++g) {
    float s = sa[g] + sb[g];
    s += __shfl_xor_sync(kFull, s, 1);
    if (MASKED && t >= valid) s = -INFINITY;
    float mx = s;
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 16));
    const float m_new = fmaxf(m[g], mx);
    alpha[g] = exp2f(m[g] - m_new);
    rescale |= (m_new != m[g]);
    m[g] = m_new;
    const float pv = exp2f(s - m_new);
    l[g] = fmaf(l[g], alpha[g], half ? 0.f : pv);
    if (!half) {
      // token t is consumed by PV group gg at step (kk - gg) mod TPG
      const int gg = t / TPG, kk = t % TPG;
      pw[g * kBlockSize + gg * TPG + (kk + TPG - gg) % TPG] = pv;
    }
  }
  __syncwarp();
  if (rescale) {  // warp-uniform: m is identical on all lanes
#pragma unroll
    for (int g = 0; g < GW; ++g)
#pragma unroll
      for (int e = 0; e < EPC; ++e) acc[g][e] *= alpha[g];
  }

  // ---- PV: lane = (chunk j, token group gg); group gg walks its tokens rotated
  // by gg so that lanes of different groups in one access phase hit different banks
  if (lane < DCH * NG) {
    const int j = lane % DCH, gg = lane / DCH;
    float pp[GW][TPG];
#pragma unroll
    for (int g = 0; g < GW; ++g) {
      const float4* src = reinterpret_cast<const float4*>(pw + g * kBlockSize + gg * TPG);
#pragma unroll
      for (int k4 = 0; k4 < TPG / 4; ++k4) {
        const float4 v = src[k4];
        pp[g][4 * k4 + 0] = v.x;
        pp[g][4 * k4 + 1] = v.y;
        pp[g][4 * k4 + 2] = v.z;
        pp[g][4 * k4 + 3] = v.w;
      }
    }
    const uint4* vcol = reinterpret_cast<const uint4*>(vt) + j;
#pragma unroll
    for (int k = 0; k < TPG; ++k) {
      const int tt = gg * TPG + ((k + gg) % TPG);
      float vf[EPC];
      Elem<T>::unpack(vcol[tt * DCH], vf);
      if (MASKED && tt >= valid) {
#pragma unroll
        for (int e = 0; e < EPC; ++e) vf[e] = 0.f;   // unused slots may hold anything
      }
#pragma unroll
      for (int g = 0; g < GW; ++g)
#pragma unroll
        for (int e = 0; e < EPC; ++e) acc[g][e] = fmaf(pp[g][k], vf[e], acc[g][e]);
    }
  }
  __syncwarp();
}

}  // namespace

template <typename T, int D, int GW, bool BALANCED>
__global__ void __launch_bounds__((kMaxConsumerWarps + 1) * 32, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                        const DecodeParams p) {
  constexpr int EPC = Elem<T>::kPerChunk;
  constexpr int DCH = D / EPC;
  constexpr int CPL = DCH / 2;
  constexpr int NG = 32 / DCH;
  static_assert(D % EPC == 0 && DCH % 2 == 0 && DCH <= 32 && kBlockSize % NG == 0, "unsupported head_dim");
  static_assert((kBlockSize / NG) % 4 == 0, "token groups must be float4-sized");

  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int32_t warp_tot[32];

  const int HG = p.heads_per_cta, WPK = p.warps_per_kv, NCW = HG * WPK, STAGES = p.stages;
  const int tile_bytes = kBlockSize * HG * D * (int)sizeof(T);
  const int stage_bytes = 2 * tile_bytes;
  float* p_buf = reinterpret_cast<float*>(smem + STAGES * stage_bytes);
  uint64_t* full_bar =
      reinterpret_cast<uint64_t*>(smem + STAGES * stage_bytes + ((NCW * GW * kBlockSize * 4 + 15) & ~15));
  uint64_t* empty_bar = full_bar + kMaxStages;
  int32_t* prefix = reinterpret_cast<int32_t*>(empty_bar + kMaxStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hg = blockIdx.y;
  const int B = p.batch;
  const int G = p.num_heads / p.num_kv_heads;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], NCW);
    }
    fence_mbar_init();
  }
  if (warp == NCW && lane == 0) {
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }

  // ---------------------------------------------------------------- work range
  int g_begin = 0, g_end = 0, b_first = 0, w_eff = 1, total = 0;
  int chunk = 0, n_split = 0;  // split schedule: chunk index and pages of the sequence
  if constexpr (BALANCED) {
    build_page_prefix(p, prefix, warp_tot);  // contains __syncthreads (also publishes the barrier init)
    total = prefix[B];
    w_eff = min((int)gridDim.x, total);
    if ((int)blockIdx.x < w_eff) {
      g_begin = (int)((int64_t)total * blockIdx.x / w_eff);
      g_end = (int)((int64_t)total * (blockIdx.x + 1) / w_eff);
      int lo = 0, hi = B;  // last b with prefix[b] <= g_begin
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= g_begin) lo = mid; else hi = mid - 1;
      }
      b_first = lo;
    }
    // rows with nothing to attend to are written as zeros
    for (int b = blockIdx.x; b < B; b += gridDim.x)
      if (prefix[b + 1] == prefix[b])
        write_zero_row<T, D>(p, b, hg * HG * G, (hg + 1) * HG * G, threadIdx.x, blockDim.x);
  } else {
    b_first = blockIdx.x / p.max_chunks;
    chunk = blockIdx.x % p.max_chunks;
    n_split = pages_of(p, b_first, chunk == 0 && hg == 0);
    g_begin = chunk * p.split_pages;
    g_end = min(n_split, g_begin + p.split_pages);
    if (n_split == 0 && chunk == 0)
      write_zero_row<T, D>(p, b_first, hg * HG * G, (hg + 1) * HG * G, threadIdx.x, blockDim.x);
    __syncthreads();
  }
  if (g_begin >= g_end) return;  // uniform over the CTA: nothing issued, nothing pending

  // ---------------------------------------------------------------- producer
  if (warp == NCW) {
    uint32_t it = 0;
    bool ok = true;
    int b = b_first, g = g_begin;
    while (g < g_end && ok) {
      int s0 = 0, s1 = n_split;
      if constexpr (BALANCED) {
        while (prefix[b + 1] <= g) ++b;
        s0 = prefix[b];
        s1 = prefix[b + 1];
      }
      const int seg_end = min(g_end, s1);
      const int32_t* row = p.block_table + (int64_t)b * p.bt_sb;
      for (int lp = g - s0; lp < seg_end - s0 && ok; lp += 32) {
        const int cnt = min(32, seg_end - s0 - lp);
        int my_page = lane < cnt ? __ldg(row + lp + lane) : 0;
        if (lane < cnt && (my_page < 0 || (int64_t)my_page >= p.num_blocks)) set_error(p.error, kErrBadPage);
        for (int i = 0; i < cnt; ++i, ++it) {
          const int page = __shfl_sync(kFull, my_page, i);
          int good = 1;
          if (lane == 0) {
            const int s = it % STAGES;
            const uint32_t ph = (it / STAGES) & 1;
            if (!mbar_wait_bounded(&empty_bar[s], ph ^ 1)) {
              good = 0;
            } else {
              mbar_arrive_expect_tx(&full_bar[s], stage_bytes);
              uint8_t* dst = smem + s * stage_bytes;
              // out-of-range pages (reported above) read as zeros: TMA fills outside the tensor
              tma_load_4d(dst, &tmap_k, 0, 0, hg * HG, page, &full_bar[s]);
              tma_load_4d(dst + tile_bytes, &tmap_v, 0, 0, hg * HG, page, &full_bar[s]);
            }
          }
          good = __shfl_sync(kFull, good, 0);
          if (!good) {
            ok = false;
            break;
          }
        }
      }
      g = seg_end;
      ++b;
    }
    if (!ok && lane == 0) set_error(p.error, kErrTimeout);
    // the CTA must not retire with bulk copies still writing its shared memory
    if (lane == 0) {
      const uint32_t n = it < (uint32_t)STAGES ? it : (uint32_t)STAGES;
      for (uint32_t k = 1; k <= n; ++k) {
        const uint32_t i = it - k;
        if (!mbar_wait_bounded(&full_bar[i % STAGES], (i / STAGES) & 1)) set_error(p.error, kErrTimeout);
      }
    }
    return;
  }
  if (warp > NCW) return;

  // ---------------------------------------------------------------- consumers
  const int kh = warp / WPK, r = warp % WPK;
  const int kvh = hg * HG + kh;
  const int head0 = kvh * G + r * GW;
  float* pw = p_buf + warp * GW * kBlockSize;
  const int t = lane >> 1, half = lane & 1;
  (void)t;

  uint32_t it = 0;
  bool first_seg = true;
  int b = b_first, g = g_begin;
  while (g < g_end) {
    int s0 = 0, s1 = n_split;
    if constexpr (BALANCED) {
      while (prefix[b + 1] <= g) ++b;
      s0 = prefix[b];
      s1 = prefix[b + 1];
    }
    const int n_b = s1 - s0;
    const int seg_end = min(g_end, s1);
    const int lp0 = g - s0, lp1 = seg_end - s0;
    const int ctx = min(max(__ldg(&p.context_lens[b]), 0), n_b * kBlockSize);

    // q of this warp's heads: this lane's half of D, prescaled into the exp2 domain
    float qv[GW][D / 2];
#pragma unroll
    for (int gq = 0; gq < GW; ++gq) {
      const uint4* qrow = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.q) + (int64_t)b * p.q_sb +
                                                         (int64_t)(head0 + gq) * p.q_sh) +
                          half * CPL;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        float f[EPC];
        Elem<T>::unpack(__ldg(qrow + c), f);
#pragma unroll
        for (int e = 0; e < EPC; ++e) qv[gq][c * EPC + e] = f[e] * p.scale_log2;
      }
    }
    float m[GW], l[GW], acc[GW][EPC];
#pragma unroll
    for (int gq = 0; gq < GW; ++gq) {
      m[gq] = -INFINITY;
      l[gq] = 0.f;
#pragma unroll
      for (int e = 0; e < EPC; ++e) acc[gq][e] = 0.f;
    }

    bool ok = true;
    for (int lp = lp0; lp < lp1; ++lp, ++it) {
      const int s = it % STAGES;
      if (!mbar_wait_bounded(&full_bar[s], (it / STAGES) & 1)) {
        ok = false;
        break;
      }
      const T* kt = reinterpret_cast<const T*>(smem + s * stage_bytes) + kh * kBlockSize * D;
      const T* vt = reinterpret_cast<const T*>(smem + s * stage_bytes + tile_bytes) + kh * kBlockSize * D;
      const int valid = ctx - lp * kBlockSize;
      if (valid >= kBlockSize)
        page_update<T, D, GW, false>(kt, vt, valid, qv, m, l, acc, pw, lane);
      else
        page_update<T, D, GW, true>(kt, vt, valid, qv, m, l, acc, pw, lane);
      if (lane == 0) mbar_arrive(&empty_bar[s]);
    }
    if (!__all_sync(kFull, ok)) {
      if (lane == 0) set_error(p.error, kErrTimeout);
      return;
    }

    // ---- segment epilogue
#pragma unroll
    for (int gq = 0; gq < GW; ++gq) l[gq] = warp_sum(l[gq]);
    if constexpr (NG > 1) {
#pragma unroll
      for (int off = (NG / 2) * DCH; off >= DCH; off /= 2)
#pragma unroll
        for (int gq = 0; gq < GW; ++gq)
#pragma unroll
          for (int e = 0; e < EPC; ++e) acc[gq][e] += __shfl_down_sync(kFull, acc[gq][e], off);
    }
    if (lp0 == 0 && lp1 == n_b) {
      if (lane < DCH) {
#pragma unroll
        for (int gq = 0; gq < GW; ++gq) {
          const float inv = 1.f / l[gq];
          float o[EPC];
#pragma unroll
          for (int e = 0; e < EPC; ++e) o[e] = acc[gq][e] * inv;
          T* dst = reinterpret_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)(head0 + gq) * p.o_sh + lane * EPC;
          *reinterpret_cast<uint4*>(dst) = Elem<T>::pack(o);
        }
      }
    } else {
      int64_t slot;
      if constexpr (BALANCED)
        slot = 2 * (int64_t)blockIdx.x + (first_seg ? 0 : 1);
      else
        slot = (int64_t)b * p.max_chunks + chunk;
      if (lane < DCH) {
#pragma unroll
        for (int gq = 0; gq < GW; ++gq) {
          float4* dst = reinterpret_cast<float4*>(p.part_o + (slot * p.num_heads + head0 + gq) * D + lane * EPC);
#pragma unroll
          for (int e4 = 0; e4 < EPC / 4; ++e4)
            dst[e4] = make_float4(acc[gq][4 * e4], acc[gq][4 * e4 + 1], acc[gq][4 * e4 + 2], acc[gq][4 * e4 + 3]);
        }
      }
      if (lane == 0) {
#pragma unroll
        for (int gq = 0; gq < GW; ++gq) p.part_ml[slot * p.num_heads + head0 + gq] = make_float2(m[gq], l[gq]);
      }
      if constexpr (BALANCED) {
        // Publish this part, count it; the warp that brings the count to the
        // number of parts merges them (and re-arms the counter for the next call).
        __threadfence();
        __syncwarp();
        const int sb0 = s0, sb1 = s1;
        auto wid = [&](int gp) { return (int)(((int64_t)(gp + 1) * w_eff - 1) / total); };
        const int w_first = wid(sb0), w_last = wid(sb1 - 1);
        const int nparts = w_last - w_first + 1;
        int last = 0;
        if (lane == 0) {
          int32_t* ctr = p.counters + (int64_t)b * (p.num_kv_heads * WPK) + kvh * WPK + r;
          const int old = atomicAdd(ctr, 1);
          last = old == nparts - 1;
          if (last) atomicExch(ctr, 0);
        }
        last = __shfl_sync(kFull, last, 0);
        if (last) {
          __threadfence();
          auto slot_of = [&](int i) -> int64_t {
            const int w = w_first + i;
            const int sw = (int)((int64_t)total * w / w_eff);
            return 2 * (int64_t)w + (sw < sb0 ? 1 : 0);
          };
#pragma unroll
          for (int gq = 0; gq < GW; ++gq) merge_parts<T, D>(p, b, head0 + gq, nparts, slot_of, lane);
        }
      }
    }
    first_seg = false;
    g = seg_end;
    ++b;
  }
}

// Split schedule: merge the chunks of every sequence that has more than one.
// One warp per (sequence, query head).
template <typename T, int D>
__global__ void __launch_bounds__(128) lse_combine_kernel(const DecodeParams p) {
  const int gw = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= p.batch * p.num_heads) return;
  const int b = gw / p.num_heads, h = gw % p.num_heads;
  const int n_b = pages_of(p, b, false);
  const int nparts = (n_b + p.split_pages - 1) / p.split_pages;
  if (nparts <= 1) return;  // the decode kernel wrote the row directly
  auto slot_of = [&](int i) -> int64_t { return (int64_t)b * p.max_chunks + i; };
  merge_parts<T, D>(p, b, h, nparts, slot_of, lane);
}

// ---------------------------------------------------------------- host side

int decode_smem_bytes(int dtype_bytes, int head_dim, int heads_per_cta, int warps_per_kv, int gw, int stages,
                      int prefix_entries) {
  const int tile = kBlockSize * heads_per_cta * head_dim * dtype_bytes;
  const int ncw = heads_per_cta * warps_per_kv;
  int bytes = stages * 2 * tile;
  bytes += (ncw * gw * kBlockSize * 4 + 15) & ~15;
  bytes += 2 * kMaxStages * 8;
  bytes += prefix_entries * 4;
  return bytes;
}

template <typename T, int D, int GW, bool BAL>
static cudaError_t launch_one(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                              const LaunchShape& s, cudaStream_t stream) {
  auto kern = paged_decode_kernel<T, D, GW, BAL>;
  // raise the dynamic shared-memory limit once per device (and when a call needs more)
  static int granted[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || granted[dev] < s.smem_bytes) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, s.smem_bytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) granted[dev] = s.smem_bytes;
  }
  kern<<<s.grid, s.block, s.smem_bytes, stream>>>(tk, tv, p);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_d(int gw, bool bal, const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p,
                            const LaunchShape& s, cudaStream_t st) {
  if (gw == 1) return bal ? launch_one<T, D, 1, true>(tk, tv, p, s, st) : launch_one<T, D, 1, false>(tk, tv, p, s, st);
  return bal ? launch_one<T, D, 2, true>(tk, tv, p, s, st) : launch_one<T, D, 2, false>(tk, tv, p, s, st);
}

template <typename T>
static cudaError_t launch_t(int head_dim, int gw, bool bal, const CUtensorMap& tk, const CUtensorMap& tv,
                            const DecodeParams& p, const LaunchShape& s, cudaStream_t st) {
  switch (head_dim) {
    case 64: return launch_d<T, 64>(gw, bal, tk, tv, p, s, st);
    case 112: return launch_d<T, 112>(gw, bal, tk, tv, p, s, st);
    case 128: return launch_d<T, 128>(gw, bal, tk, tv, p, s, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_paged_decode(int dtype, int head_dim, int gw, bool balanced, const CUtensorMap& tmap_k,
                                const CUtensorMap& tmap_v, const DecodeParams& p, const LaunchShape& shape,
                                cudaStream_t stream) {
  switch (dtype) {
    case UBX_DTYPE_F32: return launch_t<float>(head_dim, gw, balanced, tmap_k, tmap_v, p, shape, stream);
    case UBX_DTYPE_BF16: return launch_t<__nv_bfloat16>(head_dim, gw, balanced, tmap_k, tmap_v, p, shape, stream);
    case UBX_DTYPE_F16: return launch_t<__half>(head_dim, gw, balanced, tmap_k, tmap_v, p, shape, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t combine_t(int head_dim, const DecodeParams& p, cudaStream_t st) {
  const int warps = p.batch * p.num_heads;
  const dim3 grid((warps + 3) / 4), block(128);
  switch (head_dim) {
    case 64: lse_combine_kernel<T, 64><<<grid, block, 0, st>>>(p); break;
    case 112: lse_combine_kernel<T, 112><<<grid, block, 0, st>>>(p); break;
    case 128: lse_combine_kernel<T, 128><<<grid, block, 0, st>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_lse_combine(int dtype, int head_dim, const DecodeParams& p, cudaStream_t stream) {
  switch (dtype) {
    case UBX_DTYPE_F32: return combine_t<float>(head_dim, p, stream);
    case UBX_DTYPE_BF16: return combine_t<__nv_bfloat16>(head_dim, p, stream);
    case UBX_DTYPE_F16: return combine_t<__half>(head_dim, p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ubx
