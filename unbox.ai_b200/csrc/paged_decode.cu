// Paged GQA decode attention for sm_100a.
//
// Semantics follow paged_decode_attention_ref
// (unbox_platform/infer/kernels/paged_decode_attention.py:157-191): for every
// sequence b and query head h, softmax(scale * q . K) V over the first
// context_lens[b] positions, position j read from page block_table[b, j / 16],
// slot j % 16, KV head h / (H / KVH).
//
// Structure (one CTA per SM, persistent):
//   * In the KVPool layout (kvcache.py:248-251) one token row of a page holds
//     all KV heads contiguously (KVH * D elements). The CTA's head group of a
//     page is 16 such rows; each is moved with one bulk copy (cp.async.bulk on
//     the TMA engine) into a shared-memory tile whose row pitch is padded to an
//     odd number of 16-byte chunks, so ldmatrix reads are bank-conflict free.
//   * Warp NCW is the producer: it walks the CTA's pages, reads the block table
//     32 entries at a time and has its 32 lanes issue the 32 row copies (16 K,
//     16 V) of every page into a ring of `stages` buffers guarded by full/empty
//     mbarriers.
//   * bf16 / fp16: consumer warp w owns KV head w of the head group with all of
//     its query heads as the rows of one tensor-core tile (mma m16n8k16 fed by
//     ldmatrix from the page tiles); QK's accumulator fragments are reused as
//     the P operand of PV, online softmax runs on them with two shuffles per row.
//   * fp32: CUDA-core consumer, warp = (KV head, <= 2 query heads): QK with two
//     lanes per token holding half of q in registers, PV with lane = (16-byte
//     chunk of D, token group).
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
#include <type_traits>

#include "ubx_cascade_prefix.cuh"
#include "ubx_common.cuh"
#include "ubx_internal.h"
#include "ubx_mma.cuh"
#include "ubx_prep.cuh"

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

// Balanced schedule: this CTA's index among the CTAs that split the page
// ranges, and their number (a fused cascade launch runs its shared-prefix CTAs
// first, at indices below p.range_first).
__device__ __forceinline__ int range_cta(const DecodeParams& p) { return (int)blockIdx.x - p.range_first; }
__device__ __forceinline__ int range_ctas(const DecodeParams& p) { return (int)gridDim.x - p.range_first; }

// prefix[b] = pages of sequences 0..b-1, prefix[B] = total. Whole CTA.
__device__ void build_page_prefix(const DecodeParams& p, int32_t* prefix, int32_t* warp_tot) {
  const int B = p.batch;
  const int nt = blockDim.x;
  const int per = (B + nt - 1) / nt;
  const int b0 = min(B, (int)threadIdx.x * per);
  const int b1 = min(B, b0 + per);
  const bool report = range_cta(p) == 0 && blockIdx.y == 0;
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
    if (p.lse && c == 0) p.lse[(int64_t)b * p.num_heads + h] = -INFINITY;  // nothing attended
  }
}

// Merge the `nparts` partial (acc, max, sum) triples of heads head0 .. head0+nh-1
// of sequence b into normalised output rows. Lanes are (head, 16-byte output
// chunk) pairs, and the loads of several parts are in flight together, so a
// merge costs a few L2 round trips rather than one per part and head.
template <typename T, int D, typename SlotFn>
__device__ void merge_rows(const DecodeParams& p, int b, int head0, int nh, int nparts, SlotFn slot_of, int lane) {
  constexpr int EPC = Elem<T>::kPerChunk;
  constexpr int DCH = D / EPC;   // output chunks per row
  constexpr int HPW = 32 / DCH;  // heads per pass of the warp
  const int H = p.num_heads;
  for (int hb = 0; hb < nh; hb += HPW) {
    const int h = hb + lane / DCH, c = lane % DCH;
    if (lane >= HPW * DCH || h >= nh) continue;  // no warp collectives below
    const int head = head0 + h;
    // one pass with a running max: all of a part's loads are independent of the
    // previous parts, so unrolled iterations keep several parts in flight
    float M = -INFINITY, L = 0.f, o[EPC];
#pragma unroll
    for (int e = 0; e < EPC; ++e) o[e] = 0.f;
    auto fold = [&](const float2 ml, const float4* src) {
      float4 v[EPC / 4];
#pragma unroll
      for (int e4 = 0; e4 < EPC / 4; ++e4) v[e4] = __ldcg(src + e4);
      if (ml.x > M) {
        const float sc = exp2f(M - ml.x);  // M = -inf at first: sc = 0
        L *= sc;
#pragma unroll
        for (int e = 0; e < EPC; ++e) o[e] *= sc;
        M = ml.x;
      }
      const float wgt = exp2f(ml.x - M);
      L = fmaf(ml.y, wgt, L);
#pragma unroll
      for (int e4 = 0; e4 < EPC / 4; ++e4) {
        o[4 * e4 + 0] = fmaf(wgt, v[e4].x, o[4 * e4 + 0]);
        o[4 * e4 + 1] = fmaf(wgt, v[e4].y, o[4 * e4 + 1]);
        o[4 * e4 + 2] = fmaf(wgt, v[e4].z, o[4 * e4 + 2]);
        o[4 * e4 + 3] = fmaf(wgt, v[e4].w, o[4 * e4 + 3]);
      }
    };
#pragma unroll 8
    for (int i = 0; i < nparts; ++i) {
      const int64_t slot = slot_of(i);
      fold(__ldcg(&p.part_ml[slot * H + head]),
           reinterpret_cast<const float4*>(p.part_o + (slot * H + head) * D + c * EPC));
    }
    const float inv = 1.f / L;
#pragma unroll
    for (int e = 0; e < EPC; ++e) o[e] *= inv;
    T* dst = reinterpret_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)head * p.o_sh + c * EPC;
    *reinterpret_cast<uint4*>(dst) = Elem<T>::pack(o);
    if (p.lse && c == 0) p.lse[(int64_t)b * H + head] = M + log2f(L);
  }
}

// One page of one KV head for the GW query heads of this warp.
//   kt, vt: this warp's KV head in the page tiles: 16 rows of D elements, row
//           stride rs elements
//   pw:     this warp's probability buffer [GW][16] (rotated per token group)
template <typename T, int D, int GW, bool MASKED>
__device__ __forceinline__ void page_update(const T* __restrict__ kt, const T* __restrict__ vt, int rs, int valid,
                                            const float (&qv)[GW][D / 2], float (&m)[GW], float (&l)[GW],
                                            float (&acc)[GW][Elem<T>::kPerChunk], float* pw, int lane) {
  constexpr int EPC = Elem<T>::kPerChunk;
  constexpr int DCH = D / EPC;       // 16-byte chunks per row
  constexpr int CPL = DCH / 2;       // QK: chunks per lane (two lanes per token)
  constexpr int NG = 32 / DCH;       // PV: token groups
  constexpr int TPG = kBlockSize / NG;
  const int t = lane >> 1, half = lane & 1;

  // ---- scores: lane pair (2t, 2t+1) covers token t, each lane half of D
  const uint4* krow = reinterpret_cast<const uint4*>(kt + t * rs) + half * CPL;
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
#pragma unroll
    for (int k = 0; k < TPG; ++k) {
      const int tt = gg * TPG + ((k + gg) % TPG);
      float vf[EPC];
      Elem<T>::unpack(reinterpret_cast<const uint4*>(vt + tt * rs)[j], vf);
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

// ---------------------------------------------------------------- shared CTA plumbing

struct Work {
  int g_begin, g_end, b_first, w_eff, total, chunk, n_split, trim;
};

// Balanced ranges: CTA x streams flattened pages [range_begin(x),
// range_begin(x + 1)). The shares are equal, except that with `trim` > 0 the
// last CTA takes `trim` pages fewer than the others: under programmatic overlap
// it is the CTA the hardware dispatches last, onto the SM that the previous
// grid's last CTA frees, so it starts after every other CTA has prefetched.
__device__ __forceinline__ int range_begin(const Work& w, int x) {
  return x >= w.w_eff ? w.total : (int)((int64_t)(w.total + w.trim) * x / w.w_eff);
}

// The CTA whose range holds flattened page gp.
__device__ __forceinline__ int cta_of(const Work& w, int gp) {
  return min(w.w_eff - 1, (int)(((int64_t)(gp + 1) * w.w_eff - 1) / (w.total + w.trim)));
}

struct Seg {
  int b, s0, s1, lp0, lp1;
};

// Position in the stage ring: the stage index and the phase parity its
// barriers are in (kept incrementally: no integer division per page).
struct RingPos {
  int st;
  uint32_t ph;
  __device__ __forceinline__ void next(int stages) {
    if (++st == stages) {
      st = 0;
      ph ^= 1u;
    }
  }
  __device__ __forceinline__ void prev(int stages) {
    if (st == 0) {
      st = stages - 1;
      ph ^= 1u;
    } else {
      --st;
    }
  }
};

struct Smem {
  uint8_t* stages;
  float* p_buf;
  uint64_t* full_bar;
  uint64_t* empty_bar;
  int32_t* prefix;
};

// Layout: [stages][p_buf][full x stages][empty x stages][prefix]
// (per-stage slots sized by the launch's stage count: every byte counts toward
// fitting one more stage)
__device__ __forceinline__ Smem carve_smem(uint8_t* smem, const DecodeParams& p) {
  Smem s;
  const int stage_bytes = 2 * p.tile_bytes;
  s.stages = smem;
  s.p_buf = reinterpret_cast<float*>(smem + p.stages * stage_bytes);
  s.full_bar = reinterpret_cast<uint64_t*>(smem + p.stages * stage_bytes + p.pbuf_bytes);
  s.empty_bar = s.full_bar + p.stages;
  s.prefix = reinterpret_cast<int32_t*>(s.empty_bar + p.stages);
  return s;
}

// Pages this CTA streams: a contiguous range of the flattened (sequence, page)
// list (balanced) or one chunk of one sequence (split). Reads only
// context_lens. Ends with a CTA barrier (publishes mbarrier init).
template <typename T, int D, bool BAL>
__device__ Work setup_work(const DecodeParams& p, const Smem& sm, int32_t* warp_tot) {
  Work w{0, 0, 0, 1, 0, 0, 0, 0};
  const int B = p.batch;
  if constexpr (BAL) {
    build_page_prefix(p, sm.prefix, warp_tot);
    w.total = sm.prefix[B];
    w.w_eff = min(range_ctas(p), w.total);
    // the last range keeps at least half of an even share
    if (w.w_eff > 1) w.trim = max(0, min(p.tail_trim, w.total / (2 * w.w_eff)));
    const int x = range_cta(p);
    if (x < w.w_eff) {
      w.g_begin = range_begin(w, x);
      w.g_end = range_begin(w, x + 1);
      int lo = 0, hi = B;  // last b with prefix[b] <= g_begin
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (sm.prefix[mid] <= w.g_begin) lo = mid; else hi = mid - 1;
      }
      w.b_first = lo;
    }
  } else {
    w.b_first = blockIdx.x / p.max_chunks;
    w.chunk = blockIdx.x % p.max_chunks;
    w.n_split = pages_of(p, w.b_first, w.chunk == 0 && blockIdx.y == 0);
    w.g_begin = w.chunk * p.split_pages;
    w.g_end = min(w.n_split, w.g_begin + p.split_pages);
    __syncthreads();
  }
  return w;
}

// Rows of sequences with nothing to attend to are written as zeros (the
// reference raises there). Runs after the grid-dependency wait: it writes `out`.
template <typename T, int D, bool BAL>
__device__ void write_zero_rows(const DecodeParams& p, const Work& w, const int32_t* prefix, int head_lo,
                                int head_hi, int tid, int nthreads) {
  if constexpr (BAL) {
    for (int b = range_cta(p); b < p.batch; b += range_ctas(p))
      if (prefix[b + 1] == prefix[b]) write_zero_row<T, D>(p, b, head_lo, head_hi, tid, nthreads);
  } else {
    if (w.n_split == 0 && w.chunk == 0) write_zero_row<T, D>(p, w.b_first, head_lo, head_hi, tid, nthreads);
  }
}

// Next (sequence, page range) segment of the CTA's work; b and g are the cursor.
template <bool BAL>
__device__ __forceinline__ bool next_seg(const Work& w, const int32_t* prefix, int& b, int& g, Seg& s) {
  if (g >= w.g_end) return false;
  if constexpr (BAL) {
    while (prefix[b + 1] <= g) ++b;
    s.s0 = prefix[b];
    s.s1 = prefix[b + 1];
  } else {
    s.s0 = 0;
    s.s1 = w.n_split;
  }
  s.b = b;
  const int seg_end = min(w.g_end, s.s1);
  s.lp0 = g - s.s0;
  s.lp1 = seg_end - s.s0;
  g = seg_end;
  ++b;
  return true;
}

// Fused KV append (whole producer warp): write the new token of sequence b --
// position context_lens[b] - 1, the engine's append at engine.py:213-215 --
// into its slot of `page` for the heads this CTA streams, then fence so the
// TMA load of the same page that follows sees the rows.
template <typename T, int D>
__device__ void append_rows(const DecodeParams& p, int b, int page, int head0, int nheads, int lane) {
  constexpr int CPR = D * (int)sizeof(T) / 16;  // 16-byte chunks per row
  const int ctx = __ldg(&p.context_lens[b]);
  // no token to place, a clamped context (reported by pages_of) or a bad page
  // (reported by the producer; the tile then reads as zeros)
  if (ctx < 1 || (ctx - 1) / kBlockSize >= p.max_blocks || page < 0 || (int64_t)page >= p.num_blocks) return;
  const int slot = (ctx - 1) % kBlockSize;
  const int per_kv = nheads * CPR;
  for (int i = lane; i < 2 * per_kv; i += 32) {
    const int which = i / per_kv, r = i % per_kv, h = head0 + r / CPR, c = r % CPR;
    const T* src = reinterpret_cast<const T*>(which ? p.v_new : p.k_new) + (int64_t)b * p.n_stok +
                   (int64_t)h * p.n_sh + c * (16 / (int)sizeof(T));
    T* dst = const_cast<T*>(reinterpret_cast<const T*>(which ? p.v_cache : p.k_cache)) + (int64_t)page * p.c_sblk +
             (int64_t)slot * p.c_stok + (int64_t)h * p.c_sh + c * (16 / (int)sizeof(T));
    *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
  }
  fence_proxy_async_global();
  __syncwarp();
}

// True when the segment ends its sequence and the fused append has a token to
// place (a clamped context has none: pages_of reported it).
__device__ __forceinline__ bool segment_appends(const DecodeParams& p, const Seg& s) {
  if (p.k_new == nullptr || s.lp1 != s.s1 - s.s0) return false;
  const int ctx = __ldg(&p.context_lens[s.b]);
  return ctx >= 1 && (ctx - 1) / kBlockSize < p.max_blocks;
}

// Producer warp: reads the block table 32 entries at a time; for every page
// lane 0 claims a free stage and the 32 lanes each issue one row copy (lanes
// 0-15 the K rows, 16-31 the V rows of the CTA's heads). With APPEND_HERE the
// producer also performs the fused KV append (CUDA-core path; the tensor-core
// consumers append themselves).
template <typename T, int D, bool BAL, bool APPEND_HERE>
__device__ void produce(const DecodeParams& p, const Work& w, const Smem& sm, int head0, int lane) {
  const int STAGES = p.stages;
  const int tile = p.tile_bytes, stage_bytes = 2 * tile;
  const char* base = reinterpret_cast<const char*>(lane < 16 ? p.k_cache : p.v_cache) +
                     (int64_t)head0 * p.c_sh * (int64_t)sizeof(T);
  const int t = lane & 15;
  const int dst_off = (lane >> 4) * tile + t * p.smem_row_bytes;
  const uint64_t stream_policy = l2_policy_evict_first();  // pages are read once: keep the metadata in L2
  uint32_t it = 0;
  RingPos pos{0, 0};
  bool ok = true;
  int b = w.b_first, g = w.g_begin;
  Seg s;
  while (ok && next_seg<BAL>(w, sm.prefix, b, g, s)) {
    const int32_t* row = p.block_table + (int64_t)s.b * p.bt_sb;
    for (int lp = s.lp0; lp < s.lp1 && ok; lp += 32) {
      const int cnt = min(32, s.lp1 - lp);
      const int my_page = lane < cnt ? __ldg(row + lp + lane) : 0;
      if (lane < cnt && (my_page < 0 || (int64_t)my_page >= p.num_blocks)) set_error(p.error, kErrBadPage);
      for (int i = 0; i < cnt; ++i, ++it, pos.next(STAGES)) {
        const int page = __shfl_sync(kFull, my_page, i);
        if (APPEND_HERE && p.k_new != nullptr && lp + i == s.s1 - s.s0 - 1)
          append_rows<T, D>(p, s.b, page, head0, p.heads_per_cta, lane);
        const bool in_pool = page >= 0 && (int64_t)page < p.num_blocks;
        const int st = pos.st;
        int good = 1;
        if (lane == 0) {
          if (!mbar_wait_bounded(&sm.empty_bar[st], pos.ph ^ 1u))
            good = 0;
          else if (in_pool)
            mbar_arrive_expect_tx(&sm.full_bar[st], 2 * kBlockSize * p.row_bytes);
        }
        if (!__shfl_sync(kFull, good, 0)) {
          ok = false;
          break;
        }
        uint8_t* dst = sm.stages + st * stage_bytes;
        if (in_pool) {
          bulk_copy_g2s_hint(dst + dst_off,
                             base + ((int64_t)page * p.c_sblk + (int64_t)t * p.c_stok) * (int64_t)sizeof(T),
                             p.row_bytes, &sm.full_bar[st], stream_policy);
        } else {
          // a page outside the pool (reported above) reads as zeros
          for (int i = lane * 16; i < stage_bytes; i += 32 * 16)
            *reinterpret_cast<uint4*>(dst + i) = make_uint4(0, 0, 0, 0);
          fence_proxy_async_smem();  // before later bulk copies refill this stage
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.full_bar[st]);
        }
      }
    }
  }
  if (!ok && lane == 0) set_error(p.error, kErrTimeout);
  // the CTA must not retire with bulk copies still writing its shared memory
  if (lane == 0) {
    const uint32_t n = it < (uint32_t)STAGES ? it : (uint32_t)STAGES;
    RingPos back = pos;
    for (uint32_t k = 1; k <= n; ++k) {
      back.prev(STAGES);
      if (!mbar_wait_bounded(&sm.full_bar[back.st], back.ph)) set_error(p.error, kErrTimeout);
    }
  }
}

// Workspace slot of a partial result.
template <bool BAL>
__device__ __forceinline__ int64_t partial_slot(const DecodeParams& p, const Work& w, int b, bool first_seg) {
  if constexpr (BAL)
    return 2 * (int64_t)range_cta(p) + (first_seg ? 0 : 1);
  else
    return (int64_t)b * p.max_chunks + w.chunk;
}

// Balanced schedule: after this warp wrote its partial rows of sequence b
// (heads head0 .. head0+nh-1), count the part; the warp that completes the
// count merges all parts and re-arms the counter. No waiting on other CTAs.
template <typename T, int D>
__device__ void publish_and_merge(const DecodeParams& p, const Work& w, const Seg& s, int64_t ctr_index, int head0,
                                  int nh, int lane) {
  // the lanes' partial stores are ordered before lane 0's release by the warp
  // barrier; the counter's acquire-release add publishes them and, for the
  // warp that completes the count, orders the other parts' stores before its loads
  __syncwarp();
  const int w_first = cta_of(w, s.s0), w_last = cta_of(w, s.s1 - 1);
  const int nparts = w_last - w_first + 1;
  int last = 0;
  if (lane == 0) last = atom_add_acq_rel_gpu(&p.counters[ctr_index], 1) == nparts - 1;
  if (__shfl_sync(kFull, last, 0)) {
    // part 0's CTA may have begun its range before the sequence (its slot 1);
    // the later parts are the first segments of their CTAs (slot 0)
    const int64_t slot_first = 2 * (int64_t)w_first + (range_begin(w, w_first) < s.s0 ? 1 : 0);
    auto slot_of = [&](int i) -> int64_t { return i == 0 ? slot_first : 2 * (int64_t)(w_first + i); };
    merge_rows<T, D>(p, s.b, head0, nh, nparts, slot_of, lane);
    // re-armed for the next launch: every part has counted, and the next grid
    // reads the counter only after this one has completed
    if (lane == 0) st_relaxed_gpu(&p.counters[ctr_index], 0);
  }
}

// ---------------------------------------------------------------- consumers

// CUDA-core consumer (used for fp32): warp = (KV head, GW query heads).
template <typename T, int D, int GW, bool BAL>
__device__ void consume_fma(const DecodeParams& p, const Work& w, const Smem& sm, int kh, int kvh, int r,
                            int lane) {
  constexpr int EPC = Elem<T>::kPerChunk;
  constexpr int DCH = D / EPC;
  constexpr int CPL = DCH / 2;
  constexpr int NG = 32 / DCH;
  const int G = p.num_heads / p.num_kv_heads;
  const int head0 = kvh * G + r * GW;
  const int warp = threadIdx.x >> 5;
  float* pw = sm.p_buf + warp * GW * kBlockSize;
  const int half = lane & 1;
  const int STAGES = p.stages, stage_bytes = 2 * p.tile_bytes;
  const int rs = p.smem_row_bytes / (int)sizeof(T);  // tile row stride (elements)

  RingPos pos{0, 0};
  bool first_seg = true;
  int b = w.b_first, g = w.g_begin;
  Seg s;
  while (next_seg<BAL>(w, sm.prefix, b, g, s)) {
    const int n_b = s.s1 - s.s0;
    const int ctx = min(max(__ldg(&p.context_lens[s.b]), 0), n_b * kBlockSize);
    float qv[GW][D / 2];
#pragma unroll
    for (int gq = 0; gq < GW; ++gq) {
      const uint4* qrow = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.q) + (int64_t)s.b * p.q_sb +
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
    for (int lp = s.lp0; lp < s.lp1; ++lp, pos.next(STAGES)) {
      const int st = pos.st;
      if (!mbar_wait_bounded(&sm.full_bar[st], pos.ph)) {
        ok = false;
        break;
      }
      const T* kt = reinterpret_cast<const T*>(sm.stages + st * stage_bytes) + kh * D;
      const T* vt = reinterpret_cast<const T*>(sm.stages + st * stage_bytes + p.tile_bytes) + kh * D;
      const int valid = ctx - lp * kBlockSize;
      if (valid >= kBlockSize)
        page_update<T, D, GW, false>(kt, vt, rs, valid, qv, m, l, acc, pw, lane);
      else
        page_update<T, D, GW, true>(kt, vt, rs, valid, qv, m, l, acc, pw, lane);
      if (lane == 0) mbar_arrive(&sm.empty_bar[st]);
    }
    if (!__all_sync(kFull, ok)) {
      if (lane == 0) set_error(p.error, kErrTimeout);
      return;
    }
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
    if (s.lp0 == 0 && s.lp1 == n_b) {
      if (lane < DCH) {
#pragma unroll
        for (int gq = 0; gq < GW; ++gq) {
          const float inv = 1.f / l[gq];
          float o[EPC];
#pragma unroll
          for (int e = 0; e < EPC; ++e) o[e] = acc[gq][e] * inv;
          T* dst = reinterpret_cast<T*>(p.out) + (int64_t)s.b * p.o_sb + (int64_t)(head0 + gq) * p.o_sh + lane * EPC;
          *reinterpret_cast<uint4*>(dst) = Elem<T>::pack(o);
        }
      }
    } else {
      const int64_t slot = partial_slot<BAL>(p, w, s.b, first_seg);
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
      if constexpr (BAL) {
        const int64_t ctr = (int64_t)s.b * (p.num_kv_heads * p.warps_per_kv) + kvh * p.warps_per_kv + r;
        publish_and_merge<T, D>(p, w, s, ctr, head0, GW, lane);
      }
    }
    first_seg = false;
  }
}

// Rotary table row of position `pos` (with `report`, flags an out-of-table
// position; its rows are then left unrotated).
__device__ __forceinline__ const float2* rope_row_of(const DecodeParams& p, int pos, bool report, bool& pos_ok) {
  pos_ok = pos >= 0 && pos < p.rope_n;
  if (!pos_ok && report) set_error(p.error, kErrBadPosition);
  return reinterpret_cast<const float2*>(p.rope + (int64_t)(pos_ok ? pos : 0) * p.rope_sp);
}

// q rows in A-fragment layout (whole warp; the 4 lanes of a quad hold a row).
template <typename T, int D>
__device__ __forceinline__ void prep_q(const DecodeParams& p, int pos, bool real_row, int qc, int lane,
                                       uint32_t (&qa)[D / 16][2]) {
  constexpr int KS = D / 16;
  const float inv_d = 1.f / (float)D;
  bool pos_ok;
  const float2* rope_row = rope_row_of(p, pos, lane == 0, pos_ok);
  // the rounded products of the norm as packed multiplies (mul2_rn: the same
  // values as rounded_square / rms_apply on each element)
  float ss = 0.f;
#pragma unroll
  for (int ks = 0; ks < KS; ++ks)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float2 sq = unpack_word<T>(mul2_rn<T>(qa[ks][h], qa[ks][h]));
      ss += sq.x + sq.y;
    }
  ss += __shfl_xor_sync(kFull, ss, 1);
  ss += __shfl_xor_sync(kFull, ss, 2);
  const float rf = rms_factor<T>(ss, inv_d, p.eps);
  const uint32_t rf2 = Elem<T>::pack2(rf, rf);
  const uint32_t* w = static_cast<const uint32_t*>(p.q_w);
#pragma unroll
  for (int ks = 0; ks < KS; ++ks)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = 8 * ks + 4 * h + qc;  // element pair index of column 16ks + 8h + 2qc
      const float2 y = unpack_word<T>(mul2_rn<T>(mul2_rn<T>(qa[ks][h], rf2), __ldg(w + j)));
      const float2 cs = pos_ok ? __ldg(rope_row + j) : make_float2(1.f, 0.f);
      const float2 o = rotate_pair(y.x, y.y, cs.x, cs.y);
      qa[ks][h] = real_row ? Elem<T>::pack2(o.x, o.y) : 0u;
    }
}

// The appended K row (whole warp; lane c < D/8 holds elements 8c..8c+7 in a_row).
template <typename T, int D>
__device__ __forceinline__ void prep_k(const DecodeParams& p, int pos, int lane, uint4& a_row) {
  constexpr int RC = D / 8;
  const float inv_d = 1.f / (float)D;
  bool pos_ok;
  const float2* rope_row = rope_row_of(p, pos, false, pos_ok);  // the q rows' call reports it
  const uint32_t xw[4] = {a_row.x, a_row.y, a_row.z, a_row.w};  // element pairs
  const bool k_lane = lane < RC;
  float ss = 0.f;
  if (k_lane) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // rounded squares (packed), summed in element order
      const float2 sq = unpack_word<T>(mul2_rn<T>(xw[i], xw[i]));
      ss += sq.x;
      ss += sq.y;
    }
  }
  ss = warp_sum(ss);
  if (k_lane) {
    const float rf = rms_factor<T>(ss, inv_d, p.eps);
    const uint32_t rf2 = Elem<T>::pack2(rf, rf);
    const uint4 wr = __ldg(static_cast<const uint4*>(p.k_w) + lane);
    const uint32_t ww[4] = {wr.x, wr.y, wr.z, wr.w};
    const float4* rp = reinterpret_cast<const float4*>(rope_row + 4 * lane);
    const float4 r01 = pos_ok ? __ldg(rp) : make_float4(1.f, 0.f, 1.f, 0.f);
    const float4 r23 = pos_ok ? __ldg(rp + 1) : make_float4(1.f, 0.f, 1.f, 0.f);
    const float cs[8] = {r01.x, r01.y, r01.z, r01.w, r23.x, r23.y, r23.z, r23.w};
    uint32_t ow[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 y = unpack_word<T>(mul2_rn<T>(mul2_rn<T>(xw[i], rf2), ww[i]));
      const float2 o = rotate_pair(y.x, y.y, cs[2 * i], cs[2 * i + 1]);
      ow[i] = Elem<T>::pack2(o.x, o.y);
    }
    a_row = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
}

// Fused pre-attention at a segment start (tensor-core path): RMSNorm and the
// rotary embedding at position `pos`, applied to this warp's q rows, held in MMA
// A-fragment layout (lane (qr, qc) holds, per k-step ks, the element pairs at
// columns 16ks + 2qc and 16ks + 8 + 2qc of row qr; the 4 lanes of a quad hold a
// whole row), and to the appended K row (lane c < D/8 holds elements 8c..8c+7).
// Same steps and rounding as qk_norm_rope_kernel (model.py:25-27, :36-48).
template <typename T, int D>
__device__ __forceinline__ void prep_rows(const DecodeParams& p, int pos, bool real_row, int qc, int lane, bool append,
                                          uint32_t (&qa)[D / 16][2], uint4& a_row) {
  prep_q<T, D>(p, pos, real_row, qc, lane, qa);
  if (append) prep_k<T, D>(p, pos, lane, a_row);  // warp-uniform
}

// Tensor-core consumer (bf16 / fp16): warp = one KV head with all G <= 8 of its
// query heads as the rows of a 16-row MMA tile (rows >= G are zero).
//   QK:  S^T[16 q x 16 tok] = Q[16 x D] K^T   (m16n8k16, K rows via ldmatrix)
//   PV:  O[16 q x D] += P[16 x 16 tok] V      (V rows via ldmatrix.trans)
// The S accumulator fragments are exactly the A fragments of P, so
// probabilities never leave registers.
template <typename T, int D, bool BAL>
__device__ void consume_mma(const DecodeParams& p, const Work& w, const Smem& sm, int kh, int kvh, int lane) {
  constexpr int KS = D / 16;                // QK k-steps
  constexpr int NT = D / 8;                 // PV n-tiles
  const int G = p.num_heads / p.num_kv_heads;
  const int head0 = kvh * G;
  const int qr = lane >> 2, qc = lane & 3;
  const bool real_row = qr < G;
  const float c = p.scale_log2;
  const int STAGES = p.stages, stage_bytes = 2 * p.tile_bytes;
  const int rs = p.smem_row_bytes / (int)sizeof(T);  // tile row stride (elements)
  // per-lane ldmatrix rows: K (x4: chunk pair x token halves), V (x4.trans: token halves x chunk pair)
  const int k_row = (((lane >> 4) & 1) * 8 + (lane & 7)) * rs + ((lane >> 3) & 1) * 8;
  const int v_row = (((lane >> 3) & 1) * 8 + (lane & 7)) * rs + ((lane >> 4) & 1) * 8;

  // Fused KV append (this warp's KV head): the token at position ctx - 1 is
  // stored to the pool and patched into the shared-memory tile of the last page
  // when that page arrives (so no cross-proxy ordering with its copy).
  constexpr int RC = D / 8;  // 16-byte chunks of one head row
  const int a_which = lane / RC, a_chunk = lane % RC;
  auto store_appended = [&](const Seg& s, int a_slot, const uint4& a_row) {
    const int page = __ldg(p.block_table + (int64_t)s.b * p.bt_sb + (s.s1 - s.s0) - 1);
    if (page >= 0 && (int64_t)page < p.num_blocks)
      *(reinterpret_cast<uint4*>(const_cast<T*>(reinterpret_cast<const T*>(a_which ? p.v_cache : p.k_cache)) +
                                 (int64_t)page * p.c_sblk + (int64_t)a_slot * p.c_stok + (int64_t)kvh * p.c_sh) +
        a_chunk) = a_row;
  };

  RingPos pos{0, 0};
  bool first_seg = true;
  int b = w.b_first, g = w.g_begin;
  Seg s;
  while (next_seg<BAL>(w, sm.prefix, b, g, s)) {
    const int n_b = s.s1 - s.s0;
    const int ctx_raw = __ldg(&p.context_lens[s.b]);
    const int ctx = min(max(ctx_raw, 0), n_b * kBlockSize);
    const bool append = segment_appends(p, s);
    const int a_slot = (ctx_raw - 1) & (kBlockSize - 1);
    uint32_t qa[KS][2];
    uint4 a_row = make_uint4(0, 0, 0, 0);
    {
      const T* qrow = reinterpret_cast<const T*>(p.q) + (int64_t)s.b * p.q_sb + (int64_t)(head0 + qr) * p.q_sh;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qa[ks][0] = real_row ? __ldg(reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 2 * qc)) : 0u;
        qa[ks][1] = real_row ? __ldg(reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 8 + 2 * qc)) : 0u;
      }
      if (append && lane < 2 * RC)
        a_row = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a_which ? p.v_new : p.k_new) +
                                                     (int64_t)s.b * p.n_stok + (int64_t)kvh * p.n_sh) + a_chunk);
      if (p.rope) prep_rows<T, D>(p, ctx_raw - 1, real_row, qc, lane, append, qa, a_row);
      if (append && lane < 2 * RC) store_appended(s, a_slot, a_row);
    }
    float m = -INFINITY, l = 0.f;
    float o[NT][2];  // rows 0..7 of the O tile (q heads); rows 8..15 are padding
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = 0.f;

    bool ok = true;
    for (int lp = s.lp0; lp < s.lp1; ++lp, pos.next(STAGES)) {
      const int st = pos.st;
      if (!mbar_wait_bounded(&sm.full_bar[st], pos.ph)) {
        ok = false;
        break;
      }
      T* kt = reinterpret_cast<T*>(sm.stages + st * stage_bytes) + kh * D;
      T* vt = reinterpret_cast<T*>(sm.stages + st * stage_bytes + p.tile_bytes) + kh * D;
      const int valid = ctx - lp * kBlockSize;
      const bool patch = append && lp == n_b - 1;
      if (patch || valid < kBlockSize) {
        // slots past the context may hold anything: zero their V rows (P is 0
        // there, but 0 * NaN would not be); then place the appended row
        for (int i = lane; i < (kBlockSize - valid) * RC; i += 32)
          *reinterpret_cast<uint4*>(vt + (valid + i / RC) * rs + (i % RC) * 8) = make_uint4(0, 0, 0, 0);
        if (patch && lane < 2 * RC)
          *reinterpret_cast<uint4*>((a_which ? vt : kt) + a_slot * rs + a_chunk * 8) = a_row;
        // order these generic-proxy writes before the bulk copy that later refills the stage
        fence_proxy_async_smem();
        __syncwarp();
      }

      // ---- scores
      float sa[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4(kt + k_row + 16 * ks, r0, r1, r2, r3);
        mma16816_top<T>(sa[0], qa[ks][0], qa[ks][1], r0, r1);
        mma16816_top<T>(sa[1], qa[ks][0], qa[ks][1], r2, r3);
      }
      // this lane's scores of row qr: tokens 2qc, 2qc+1, 8+2qc, 9+2qc
      float sv[4] = {sa[0][0], sa[0][1], sa[1][0], sa[1][1]};
      if (valid < kBlockSize) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if ((i >> 1) * 8 + 2 * qc + (i & 1) >= valid) sv[i] = -INFINITY;
      }
      float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
      const float m_new = fmaxf(m, mx);
      if (__any_sync(kFull, m_new != m)) {  // rescale only when some row's max moved
        const float alpha = exp2f((m - m_new) * c);
        l *= alpha;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          o[n][0] *= alpha;
          o[n][1] *= alpha;
        }
        m = m_new;
      }
      const float mc = m * c;
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pv[i] = exp2f(fmaf(sv[i], c, -mc));
        l += pv[i];
      }
      const uint32_t pa0 = Elem<T>::pack2(pv[0], pv[1]);
      const uint32_t pa2 = Elem<T>::pack2(pv[2], pv[3]);

      // ---- PV
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4_trans(vt + v_row + 16 * np, r0, r1, r2, r3);
        mma16816_top<T>(o[2 * np], pa0, pa2, r0, r1);
        mma16816_top<T>(o[2 * np + 1], pa0, pa2, r2, r3);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty_bar[st]);
    }
    if (!__all_sync(kFull, ok)) {
      if (lane == 0) set_error(p.error, kErrTimeout);
      return;
    }

    // ---- segment epilogue (row qr lives in lanes 4qr .. 4qr+3)
    l += __shfl_xor_sync(kFull, l, 1);
    l += __shfl_xor_sync(kFull, l, 2);
    if (s.lp0 == 0 && s.lp1 == n_b) {
      if (real_row) {
        const float inv = 1.f / l;
        uint32_t* dst = reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(p.out) + (int64_t)s.b * p.o_sb +
                                                    (int64_t)(head0 + qr) * p.o_sh + 2 * qc);
#pragma unroll
        for (int n = 0; n < NT; ++n) dst[4 * n] = Elem<T>::pack2(o[n][0] * inv, o[n][1] * inv);
        if (p.lse && qc == 0) p.lse[(int64_t)s.b * p.num_heads + head0 + qr] = fmaf(m, c, log2f(l));
      }
    } else {
      const int64_t slot = partial_slot<BAL>(p, w, s.b, first_seg);
      if (real_row) {
        float2* dst = reinterpret_cast<float2*>(p.part_o + (slot * p.num_heads + head0 + qr) * D + 2 * qc);
#pragma unroll
        for (int n = 0; n < NT; ++n) dst[4 * n] = make_float2(o[n][0], o[n][1]);
        if (qc == 0) p.part_ml[slot * p.num_heads + head0 + qr] = make_float2(m * c, l);
      }
      if constexpr (BAL) publish_and_merge<T, D>(p, w, s, (int64_t)s.b * p.num_kv_heads + kvh, head0, G, lane);
    }
    first_seg = false;
  }
}

}  // namespace

// ---------------------------------------------------------------- kernels

template <typename T, int D, int GW, bool BAL>
__global__ void __launch_bounds__((kMaxConsumerWarps + 1) * 32, 1)
    paged_decode_fma_kernel(const DecodeParams p) {
  static_assert((kBlockSize / (32 / (D / Elem<T>::kPerChunk))) % 4 == 0, "token groups must be float4-sized");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ int32_t warp_tot[32];
  const Smem sm = carve_smem(smem_raw, p);
  const int HG = p.heads_per_cta, WPK = p.warps_per_kv, NCW = HG * WPK;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.num_heads / p.num_kv_heads;
  if (threadIdx.x == 0) {
    griddep_launch_dependents();  // the next grid may start on SMs this one frees
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&sm.full_bar[s], 1);
      mbar_init(&sm.empty_bar[s], NCW);
    }
    fence_mbar_init();
  }
  const Work w = setup_work<T, D, BAL>(p, sm, warp_tot);
  const bool has_work = w.g_begin < w.g_end;
  if (!has_work || warp < NCW) {
    griddep_wait();  // everything below may touch memory the previous grid wrote
    write_zero_rows<T, D, BAL>(p, w, sm.prefix, blockIdx.y * HG * G, (blockIdx.y + 1) * HG * G, threadIdx.x,
                               has_work ? NCW * 32 : blockDim.x);
  }
  if (!has_work) return;
  if (warp == NCW) {
    // the fused append in this producer reads k_new: wait for the previous grid too
    griddep_wait();
    produce<T, D, BAL, true>(p, w, sm, blockIdx.y * HG, lane);
    return;
  }
  if (warp > NCW) return;
  const int kh = warp / WPK;
  consume_fma<T, D, GW, BAL>(p, w, sm, kh, blockIdx.y * HG + kh, warp % WPK, lane);
}

// One CTA of the tensor-core decode (16-bit pools): 8 consumer warps, one per
// KV head of the CTA's head group, and a producer warp.
template <typename T, int D, bool BAL>
__device__ __forceinline__ void decode_mma_cta(const DecodeParams& p, uint8_t* smem_raw) {
  __shared__ int32_t warp_tot[32];
  const Smem sm = carve_smem(smem_raw, p);
  const int HG = p.heads_per_cta, NCW = HG;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.num_heads / p.num_kv_heads;
  if (threadIdx.x == 0) {
    griddep_launch_dependents();  // the next grid may start on SMs this one frees
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&sm.full_bar[s], 1);
      mbar_init(&sm.empty_bar[s], NCW);
    }
    fence_mbar_init();
  }
  const Work w = setup_work<T, D, BAL>(p, sm, warp_tot);
  const bool has_work = w.g_begin < w.g_end;
  if (!has_work || warp < NCW) {
    griddep_wait();  // everything below may touch memory the previous grid wrote
    write_zero_rows<T, D, BAL>(p, w, sm.prefix, blockIdx.y * HG * G, (blockIdx.y + 1) * HG * G, threadIdx.x,
                               has_work ? NCW * 32 : blockDim.x);
  }
  if (!has_work) return;
  if (warp == NCW) {
    // Streams pool pages without waiting for the previous grid: a caller that
    // launches with programmatic overlap promises that grid writes neither the
    // pool, the block table nor context_lens.
    produce<T, D, BAL, false>(p, w, sm, blockIdx.y * HG, lane);
    return;
  }
  if (warp > NCW) return;
  consume_mma<T, D, BAL>(p, w, sm, warp, blockIdx.y * HG + warp, lane);}

template <typename T, int D, bool BAL>
__global__ void __launch_bounds__((kMaxConsumerWarps + 1) * 32, 1)
    paged_decode_mma_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  decode_mma_cta<T, D, BAL>(p, smem_raw);
}

// Shared-prefix role of a fused cascade launch: CTA x (x < nctas) runs the
// (work item, KV head) pairs x, x + nctas, x + 2 nctas, ... of cp on the
// tensor cores as two independent 128-thread pipelines (warps 0-3 take every
// other pair, warps 4-7 the rest; each with its own shared-memory tiles,
// mbarriers, 256 tensor-memory columns and named barrier), so that one
// pipeline's loads and softmax overlap the other's. The ninth warp leaves.
template <typename T, int D>
__device__ void prefix_role(const CascadeParams& cp, int nctas, uint8_t* smem) {
  constexpr int GT = kTcThreads;  // threads of one pipeline
  const int tid = threadIdx.x;
  if (tid >= 2 * GT) return;
  const int grp = tid / GT, gtid = tid % GT;
  const PrefixSmem sm = carve_prefix_smem<D>(smem + grp * prefix_item_smem_bytes<D>());
  uint32_t* tmem_slot = carve_prefix_smem<D>(smem).tmem_slot;  // one allocation for both pipelines
  if (tid < 32) tc::tmem_alloc(tmem_slot, 2 * kTcCols);
  if (gtid == 0) {
    mbar_init(&sm.bar[0], 1);
    mbar_init(&sm.bar[1], 1);
    mbar_init(&sm.bar[2], 1);
    fence_mbar_init();
  }
  tc::fence_before_thread_sync();
  asm volatile("bar.sync 1, %0;" ::"n"(2 * GT) : "memory");
  tc::fence_after_thread_sync();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem = tmem_base + grp * kTcCols;
  auto sync = [grp] {
    if (grp == 0)
      asm volatile("bar.sync 2, %0;" ::"n"(GT) : "memory");
    else
      asm volatile("bar.sync 3, %0;" ::"n"(GT) : "memory");
  };
  const int pairs = cp.num_work * cp.num_kv_heads;
  uint32_t parity = 0;
  for (int i = blockIdx.x + grp * nctas; i < pairs; i += 2 * nctas)
    prefix_item<T, D>(cp, i / cp.num_kv_heads, i % cp.num_kv_heads, sm, tmem, parity, gtid, sync);
  tc::fence_before_thread_sync();
  asm volatile("bar.sync 1, %0;" ::"n"(2 * GT) : "memory");  // both pipelines are done with tensor memory
  if (tid < 32) {
    tc::fence_after_thread_sync();
    tc::tmem_dealloc(tmem_base, 2 * kTcCols);
  }
}

// Fused cascade launch, one CTA per SM: CTAs [0, p.range_first) attend every
// prefix group over its shared pages (prefix_role), CTAs [p.range_first,
// gridDim.x) stream every request's suffix pages with the balanced schedule
// (KV append fused, log-sum-exp out), side by side on disjoint SMs;
// cascade_merge_kernel follows.
template <typename T, int D>
__global__ void __launch_bounds__((kMaxConsumerWarps + 1) * 32, 1)
    cascade_fused_kernel(const DecodeParams p, const __grid_constant__ CascadeParams cp) {
  extern __shared__ __align__(128) uint8_t smem_fused[];
  if ((int)blockIdx.x < p.range_first) {
    griddep_launch_dependents();
    prefix_role<T, D>(cp, p.range_first, smem_fused);
    return;
  }
  decode_mma_cta<T, D, true>(p, smem_fused);
}

// Split schedule: merge the chunks of every sequence that has more than one.
// One CTA per (sequence, query head). Thread (chunk c, group j) folds parts
// j, j + PG, j + 2 PG, ... of 16-byte output chunk c with a running max, so
// the loads of all parts are in flight at once across the CTA; the PG groups'
// (max, sum, accumulator) are then combined through shared memory with
// log-sum-exp weights.
constexpr int kCombineThreads = 256;

template <typename T, int D>
__global__ void __launch_bounds__(kCombineThreads) lse_combine_kernel(const DecodeParams p) {
  constexpr int EPC = Elem<T>::kPerChunk;
  constexpr int DCH = D / EPC;                    // output chunks of one row
  constexpr int PG = kCombineThreads / DCH;       // part groups
  __shared__ float s_m[PG][DCH], s_l[PG][DCH];
  __shared__ float4 s_o[PG][DCH][EPC / 4];
  const int b = blockIdx.x / p.num_heads, h = blockIdx.x % p.num_heads;
  const int n_b = pages_of(p, b, false);
  const int nparts = (n_b + p.split_pages - 1) / p.split_pages;
  if (nparts <= 1) return;  // the decode kernel wrote the row directly
  const int c = threadIdx.x % DCH, j = threadIdx.x / DCH;
  if (j < PG) {
    float M = -INFINITY, L = 0.f, o[EPC];
#pragma unroll
    for (int e = 0; e < EPC; ++e) o[e] = 0.f;
#pragma unroll 4
    for (int i = j; i < nparts; i += PG) {
      const int64_t slot = (int64_t)b * p.max_chunks + i;
      const float2 ml = __ldcg(&p.part_ml[slot * p.num_heads + h]);
      const float4* src = reinterpret_cast<const float4*>(p.part_o + (slot * p.num_heads + h) * D + c * EPC);
      float4 v[EPC / 4];
#pragma unroll
      for (int e4 = 0; e4 < EPC / 4; ++e4) v[e4] = __ldcg(src + e4);
      if (ml.x > M) {
        const float sc = exp2f(M - ml.x);  // M = -inf at first: sc = 0
        L *= sc;
#pragma unroll
        for (int e = 0; e < EPC; ++e) o[e] *= sc;
        M = ml.x;
      }
      const float wgt = exp2f(ml.x - M);
      L = fmaf(ml.y, wgt, L);
#pragma unroll
      for (int e4 = 0; e4 < EPC / 4; ++e4) {
        o[4 * e4 + 0] = fmaf(wgt, v[e4].x, o[4 * e4 + 0]);
        o[4 * e4 + 1] = fmaf(wgt, v[e4].y, o[4 * e4 + 1]);
        o[4 * e4 + 2] = fmaf(wgt, v[e4].z, o[4 * e4 + 2]);
        o[4 * e4 + 3] = fmaf(wgt, v[e4].w, o[4 * e4 + 3]);
      }
    }
    s_m[j][c] = M;
    s_l[j][c] = L;
#pragma unroll
    for (int e4 = 0; e4 < EPC / 4; ++e4)
      s_o[j][c][e4] = make_float4(o[4 * e4], o[4 * e4 + 1], o[4 * e4 + 2], o[4 * e4 + 3]);
  }
  __syncthreads();
  if (threadIdx.x >= DCH) return;
  float M = -INFINITY;
  for (int g = 0; g < PG; ++g) M = fmaxf(M, s_m[g][c]);  // groups without parts hold -inf, 0
  float L = 0.f, o[EPC];
#pragma unroll
  for (int e = 0; e < EPC; ++e) o[e] = 0.f;
  for (int g = 0; g < PG; ++g) {
    const float wgt = s_m[g][c] == -INFINITY ? 0.f : exp2f(s_m[g][c] - M);
    L = fmaf(s_l[g][c], wgt, L);
#pragma unroll
    for (int e4 = 0; e4 < EPC / 4; ++e4) {
      const float4 v = s_o[g][c][e4];
      o[4 * e4 + 0] = fmaf(wgt, v.x, o[4 * e4 + 0]);
      o[4 * e4 + 1] = fmaf(wgt, v.y, o[4 * e4 + 1]);
      o[4 * e4 + 2] = fmaf(wgt, v.z, o[4 * e4 + 2]);
      o[4 * e4 + 3] = fmaf(wgt, v.w, o[4 * e4 + 3]);
    }
  }
  const float inv = 1.f / L;
#pragma unroll
  for (int e = 0; e < EPC; ++e) o[e] *= inv;
  T* dst = reinterpret_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)h * p.o_sh + c * EPC;
  *reinterpret_cast<uint4*>(dst) = Elem<T>::pack(o);
  if (p.lse && c == 0) p.lse[(int64_t)b * p.num_heads + h] = M + log2f(L);
}

// ---------------------------------------------------------------- host side

int decode_smem_bytes(int tile_bytes, int pbuf_bytes, int stages, int prefix_entries) {
  return stages * (2 * tile_bytes + kStageSlotBytes) + pbuf_bytes + prefix_entries * 4;
}

template <typename Kern>
static cudaError_t launch_with_smem(Kern kern, int* granted, const DecodeParams& p, const LaunchShape& s,
                                   cudaStream_t stream) {
  // s.overlap: programmatic dependent launch (the kernel may start while the
  // previous kernel on the stream drains; see paged_decode_mma_kernel)
  // raise the dynamic shared-memory limit once per device (and when a call needs more)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || granted[dev] < s.smem_bytes) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, s.smem_bytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) granted[dev] = s.smem_bytes;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = s.grid;
  cfg.blockDim = s.block;
  cfg.dynamicSmemBytes = s.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = s.overlap ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T, int D, int GW, bool BAL>
static cudaError_t launch_fma(const DecodeParams& p, const LaunchShape& s, cudaStream_t st) {
  static int granted[64] = {0};
  return launch_with_smem(paged_decode_fma_kernel<T, D, GW, BAL>, granted, p, s, st);
}

template <typename T, int D, bool BAL>
static cudaError_t launch_mma(const DecodeParams& p, const LaunchShape& s, cudaStream_t st) {
  static int granted[64] = {0};
  return launch_with_smem(paged_decode_mma_kernel<T, D, BAL>, granted, p, s, st);
}

template <typename T, int D>
static cudaError_t launch_d(int gw, bool bal, const DecodeParams& p, const LaunchShape& s, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    return bal ? launch_mma<T, D, true>(p, s, st) : launch_mma<T, D, false>(p, s, st);
  } else {
    if (gw == 1) return bal ? launch_fma<T, D, 1, true>(p, s, st) : launch_fma<T, D, 1, false>(p, s, st);
    return bal ? launch_fma<T, D, 2, true>(p, s, st) : launch_fma<T, D, 2, false>(p, s, st);
  }
}

template <typename T>
static cudaError_t launch_t(int head_dim, int gw, bool bal, const DecodeParams& p, const LaunchShape& s,
                            cudaStream_t st) {
  switch (head_dim) {
    case 64: return launch_d<T, 64>(gw, bal, p, s, st);
    case 112: return launch_d<T, 112>(gw, bal, p, s, st);
    case 128: return launch_d<T, 128>(gw, bal, p, s, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, int D>
static cudaError_t launch_fused_d(const DecodeParams& p, const CascadeParams& cp, const LaunchShape& s,
                                  cudaStream_t stream) {
  static int granted[64] = {0};
  auto kern = cascade_fused_kernel<T, D>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || granted[dev] < s.smem_bytes) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, s.smem_bytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) granted[dev] = s.smem_bytes;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = s.grid;
  cfg.blockDim = s.block;
  cfg.dynamicSmemBytes = s.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = s.overlap ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, kern, p, cp);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_fused_t(int head_dim, const DecodeParams& p, const CascadeParams& cp,
                                  const LaunchShape& s, cudaStream_t stream) {
  switch (head_dim) {
    case 64: return launch_fused_d<T, 64>(p, cp, s, stream);
    case 112: return launch_fused_d<T, 112>(p, cp, s, stream);
    case 128: return launch_fused_d<T, 128>(p, cp, s, stream);
    default: return cudaErrorInvalidValue;
  }
}

int fused_prefix_smem_bytes(int head_dim) {
  switch (head_dim) {
    case 64: return 2 * prefix_item_smem_bytes<64>();
    case 112: return 2 * prefix_item_smem_bytes<112>();
    case 128: return 2 * prefix_item_smem_bytes<128>();
    default: return 1 << 30;
  }
}

cudaError_t launch_cascade_fused(int dtype, int head_dim, const DecodeParams& p, const CascadeParams& cp,
                                 const LaunchShape& shape, cudaStream_t stream) {
  switch (dtype) {
    case UBX_DTYPE_BF16: return launch_fused_t<__nv_bfloat16>(head_dim, p, cp, shape, stream);
    case UBX_DTYPE_F16: return launch_fused_t<__half>(head_dim, p, cp, shape, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_paged_decode(int dtype, int head_dim, int gw, bool balanced, const DecodeParams& p,
                                const LaunchShape& shape, cudaStream_t stream) {
  switch (dtype) {
    case UBX_DTYPE_F32: return launch_t<float>(head_dim, gw, balanced, p, shape, stream);
    case UBX_DTYPE_BF16: return launch_t<__nv_bfloat16>(head_dim, gw, balanced, p, shape, stream);
    case UBX_DTYPE_F16: return launch_t<__half>(head_dim, gw, balanced, p, shape, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t combine_t(int head_dim, const DecodeParams& p, cudaStream_t st) {
  const dim3 grid((unsigned)p.batch * (unsigned)p.num_heads), block(kCombineThreads);
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
