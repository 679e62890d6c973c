// One shared-prefix work item of the cascade on the 5th-generation tensor cores
// (sm_100a): the attention of up to 128 (member request, query head) rows of a
// prefix group over a run of up to 64 shared pages of one KV head, taken 8
// pages (128 tokens) at a time with an online softmax, written as one
// unnormalised partial row per (member, head) with its (max, sum). Used by the
// standalone prefix kernel (one item per CTA, cascade.cu) and by the fused
// cascade kernel (two item pipelines in each CTA that does not stream suffix
// pages, paged_decode.cu).
//
// The reference reads shared radix-prefix pages once per request
// (unbox_platform/infer/kvcache.py:97-122 hands the requests the same pages;
// kernels/paged_decode_attention.py:157-191 attends each request over them);
// here they are loaded once per group of up to 128 rows.
#pragma once

#include <type_traits>

#include "ubx_common.cuh"
#include "ubx_internal.h"
#include "ubx_tcgen05.cuh"

namespace ubx {

constexpr int kTcRows = kCascadeRows;             // M of both MMAs: (member, query head) rows
constexpr int kTcTokens = kCascadeMaxPages * 16;  // tokens of one chunk: N of S, K of O (at most)
constexpr uint32_t kTcCols = 256;                 // TMEM of one pipeline: S (128 columns) + O (head_dim <= 128)
constexpr int kTcThreads = 128;                   // one thread per tile row
// A row's running max (log2 units) is kept while a new chunk's max exceeds it by
// at most this much: the probabilities then stay below 2^8 and the accumulator
// in tensor memory is rescaled only when the max rises further.
constexpr float kRescaleSlack = 8.f;

// Shared-memory layout of one pipeline (SWIZZLE_NONE canonical layout: a tile of
// R rows x C 16-byte chunks is stored chunk-major, [chunk][row][16 B], so 8
// consecutive rows of one chunk form a contiguous 128-byte core matrix):
//   Q [D/8][128 rows][16 B]       rows = (member, query head), member-major
//   K [D/8][128 tokens][16 B]     P [16 token chunks][128 rows][16 B] over K once S is done
//   (gap: P needs 32 KB)
//   V [D/8][128 tokens][16 B]
//   tail: 3 mbarriers, the TMEM address, the item's page ids and member sequences
// The partial rows are staged over Q, K and V at the end (rows of D floats + 16 B).
template <int D>
struct PrefixLayout {
  static constexpr int kTile = (D / 8) * kTcRows * 16;  // one operand tile
  static constexpr int kQ = 0;
  static constexpr int kK = kTile;                       // P starts here too
  static constexpr int kV = kK + (kTile > 32768 ? kTile : 32768);
  static constexpr int kTail = kV + kTile;
  static constexpr int kTailBytes = 64 + kCascadeMaxItemPages * 4 + kTcRows * 4;
  static constexpr int kBytes = (kTail + kTailBytes + 127) / 128 * 128;
  static_assert(kTcRows * (D * 4 + 16) <= kTail, "partial rows must fit over the operand tiles");
};

template <int D>
constexpr int prefix_item_smem_bytes() {
  return PrefixLayout<D>::kBytes;
}

struct PrefixSmem {
  uint8_t* base;
  uint64_t* bar;       // [3]: S complete, O complete, K and V tiles landed (tensor-map copies)
  uint32_t* tmem_slot;
  int32_t* pg_s;       // [kCascadeMaxItemPages]
  int32_t* mem_s;      // [kTcRows]
};

template <int D>
__device__ __forceinline__ PrefixSmem carve_prefix_smem(uint8_t* smem) {
  using L = PrefixLayout<D>;
  PrefixSmem s;
  s.base = smem;
  s.bar = reinterpret_cast<uint64_t*>(smem + L::kTail);
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.bar + 3);
  s.pg_s = reinterpret_cast<int32_t*>(smem + L::kTail + 64);
  s.mem_s = s.pg_s + kCascadeMaxItemPages;
  return s;
}

// Work item `wi` of p.work for KV head kvh on kTcThreads threads (tid = 0 ..
// 127, one per tile row) that synchronise with sync(). The caller owns `tmem`
// (kTcCols columns) and the three mbarriers of `sm`, initialised with one
// arrival each; `parity` is the phase they are in, advanced here once per chunk.
// With p.use_tma the K and V tiles come by tensor-map copies (p must then live
// in kernel parameter space: a __grid_constant__ argument), else by cp.async. The
// first chunk's pages are requested before griddepcontrol.wait, q and the
// partial rows are touched after it. Ends with sync(): the next item may reuse
// the shared memory and the tensor memory at once. Returns false, with the
// barriers untouched, for an item out of range (reported in the error word).
template <typename T, int D, typename Sync>
__device__ bool prefix_item(const CascadeParams& p, int wi, int kvh, const PrefixSmem& sm, uint32_t tmem,
                            uint32_t& parity, int tid, Sync sync) {
  using L = PrefixLayout<D>;
  constexpr int CH = D / 8;  // 16-byte chunks of a head row
  constexpr int R = kTcRows, TT = kTcTokens, NTH = kTcThreads;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  uint8_t* q_s = sm.base + L::kQ;
  uint8_t* k_s = sm.base + L::kK;
  uint8_t* p_s = sm.base + L::kK;
  uint8_t* v_s = sm.base + L::kV;
  const int warp = tid >> 5, lane = tid & 31;
  const int32_t* item = p.work + kCascadeWorkInts * wi;
  const int m_off = __ldg(item + 0), n_mem = __ldg(item + 1), pg_off = __ldg(item + 2), n_pg = __ldg(item + 3),
            part = __ldg(item + 4);
  const int G = p.num_heads / p.num_kv_heads;
  if (n_pg < 1 || n_pg > kCascadeMaxItemPages || n_mem < 1 || n_mem * G > R || part < 0 || part >= p.max_chunks) {
    griddep_wait();
    if (tid == 0) set_error(p.error, kErrBadWork);
    return false;  // item-uniform: every thread leaves here
  }
  // the item's page ids and member sequences, read once (plan arrays)
  for (int i = tid; i < n_pg; i += NTH) sm.pg_s[i] = __ldg(&p.page_list[pg_off + i]);
  for (int i = tid; i < n_mem; i += NTH) sm.mem_s[i] = __ldg(&p.member_list[m_off + i]);
  sync();

  // K and V of chunk c (pages 8c ..) into the tiles' canonical layout. Tensor
  // maps: one box per (page, 16-byte chunk column) -- 16 tokens x 16 bytes --
  // counted on bar[2]. cp.async: 16-byte pieces, 8 consecutive threads = 8
  // consecutive tokens of one 16-byte chunk (one core matrix). A page outside
  // the pool reads as zeros.
  bool bad_page = false;
  auto load_kv = [&](int c, int nt) {
    const int npg = nt / 16;
    if (p.use_tma) {
      if (tid == 0) {
        int valid = 0;
        for (int i = 0; i < npg; ++i) {
          const int page = sm.pg_s[c * kCascadeMaxPages + i];
          valid += page >= 0 && (int64_t)page < p.num_blocks;
        }
        mbar_arrive_expect_tx(&sm.bar[2], (uint32_t)(valid * 2 * CH * 256));
      }
      sync();  // the byte count is posted before any box can land
      for (int j = tid; j < npg * 2 * CH; j += NTH) {
        const int pc = j / (2 * CH), is_v = (j / CH) & 1, cc = j % CH;
        uint8_t* dst = (is_v ? v_s : k_s) + (cc * TT + pc * 16) * 16;
        const int page = sm.pg_s[c * kCascadeMaxPages + pc];
        if (page >= 0 && (int64_t)page < p.num_blocks) {
          tma_load_3d(dst, is_v ? &p.tmap_v : &p.tmap_k, 0, kvh * CH + cc, page * 16, &sm.bar[2]);
        } else {
          if (cc == 0 && !is_v) bad_page = true;
#pragma unroll
          for (int r = 0; r < 16; ++r) reinterpret_cast<uint4*>(dst)[r] = make_uint4(0, 0, 0, 0);
        }
      }
      return;
    }
    for (int v = tid; v < 2 * nt * CH; v += NTH) {
      const int is_v = v >= nt * CH;
      const int u = is_v ? v - nt * CH : v;
      const int t = (u / (8 * CH)) * 8 + (u & 7), cc = (u >> 3) % CH;
      uint8_t* dst = (is_v ? v_s : k_s) + (cc * TT + t) * 16;
      const int page = sm.pg_s[c * kCascadeMaxPages + (t >> 4)];
      if (page >= 0 && (int64_t)page < p.num_blocks) {
        const uint8_t* src = static_cast<const uint8_t*>(is_v ? p.v_cache : p.k_cache) +
                             ((int64_t)page * p.c_sblk + (int64_t)(t & 15) * p.c_stok + (int64_t)kvh * D) *
                                 sizeof(T) + cc * 16;
        cp_async_16(dst, src);
      } else {
        if ((t & 15) == 0 && cc == 0 && !is_v) bad_page = true;
        *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
    }
  };
  const int n_chunks = (n_pg + kCascadeMaxPages - 1) / kCascadeMaxPages;
  load_kv(0, min(n_pg, kCascadeMaxPages) * 16);
  griddep_wait();  // the first chunk's copies stay in flight across the wait
  // ---- Q rows: row r = (member r / G, query head kvh * G + r % G); rows past
  // the members are zero
  for (int v = tid; v < R * CH; v += NTH) {
    const int r = (v / (8 * CH)) * 8 + (v & 7), cc = (v >> 3) % CH;
    uint8_t* dst = q_s + (cc * R + r) * 16;
    const int mi = r / G;
    const int b = mi < n_mem ? sm.mem_s[mi] : -1;
    if (b >= 0 && b < p.batch) {
      cp_async_16(dst, static_cast<const uint8_t*>(p.q) +
                           ((int64_t)b * p.q_sb + (int64_t)(kvh * G + r % G) * p.q_sh) * sizeof(T) + cc * 16);
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  const uint32_t tmem_s = tmem, tmem_o = tmem + TT;  // columns [0, 128) and [128, 128 + D)
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const int row = warp * 32 + lane;  // this thread's tile row = TMEM lane
  const float cs = p.scale_log2;
  float m_run = -INFINITY, l_run = 0.f;  // running max (log2 units) and sum of this row
  bool ok = true;
  for (int c = 0; c < n_chunks; ++c) {
    const int NT = min(n_pg - c * kCascadeMaxPages, kCascadeMaxPages) * 16;  // tokens: N of S, K of O
    if (c > 0) load_kv(c, NT);  // the previous chunk's O = P V has completed: P (over K) and V are free
    cp_async_commit_wait_all();
    if (p.use_tma) ok = mbar_wait_bounded(&sm.bar[2], parity) && ok;
    fence_proxy_async_smem();  // these generic-proxy writes before the MMAs' reads
    tc::fence_before_thread_sync();
    sync();
    tc::fence_after_thread_sync();

    // ---- S = Q K^T (M = 128 rows, N = NT tokens, K = D): A and B K-major
    if (tid == 0) {
      const uint32_t idesc = tc::instr_desc_f16(kBf16, R, NT, false, false);
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks)
        tc::mma_f16(tmem_s, tc::smem_desc(q_s + ks * 2 * R * 16, R * 16, 128),
                    tc::smem_desc(k_s + ks * 2 * TT * 16, TT * 16, 128), idesc, ks > 0);
      tc::commit(&sm.bar[0]);
    }
    ok = mbar_wait_bounded(&sm.bar[0], parity) && ok;
    tc::fence_after_thread_sync();

    // ---- online softmax of this row: the chunk's max (first pass over tensor
    // memory), the running max and the accumulator's rescale, then the
    // probabilities (second pass)
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < TT / 16; ++j) {
      if (j * 16 < NT) {
        float v16[16];
        tc::ld16(tmem_s + lane_off + j * 16, v16);
#pragma unroll
        for (int i = 0; i < 16; ++i) mx = fmaxf(mx, v16[i]);
      }
    }
    const float mc = mx * cs;
    if (c == 0) {
      m_run = mc;
    } else {
      const bool resc = mc > m_run + kRescaleSlack;
      if (__any_sync(0xffffffffu, resc)) {  // tensor-memory accesses are warp-wide
        const float alpha = resc ? exp2f(m_run - mc) : 1.f;
#pragma unroll
        for (int j = 0; j < D / 8; ++j) {
          float o8[8];
          tc::ld8(tmem_o + lane_off + j * 8, o8);
#pragma unroll
          for (int i = 0; i < 8; ++i) o8[i] *= alpha;
          tc::st8(tmem_o + lane_off + j * 8, o8);
        }
        l_run *= alpha;
      }
      if (resc) m_run = mc;
    }
#pragma unroll
    for (int j = 0; j < TT / 16; ++j) {
      if (j * 16 < NT) {
        float v16[16];
        tc::ld16(tmem_s + lane_off + j * 16, v16);
#pragma unroll
        for (int k8 = 0; k8 < 2; ++k8) {
          float pv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            pv[i] = exp2f(fmaf(v16[k8 * 8 + i], cs, -m_run));
            l_run += pv[i];
          }
          *reinterpret_cast<uint4*>(p_s + ((2 * j + k8) * R + row) * 16) = Elem<T>::pack(pv);
        }
      }
    }
    fence_proxy_async_smem();
    tc::fence_before_thread_sync();
    sync();
    tc::fence_after_thread_sync();

    // ---- O (+)= P V (M = 128 rows, N = D, K = NT tokens): P K-major, V MN-major
    if (tid == 0) {
      const uint32_t idesc = tc::instr_desc_f16(kBf16, R, D, false, true);
      for (int ks = 0; ks < NT / 16; ++ks)
        tc::mma_f16(tmem_o, tc::smem_desc(p_s + ks * 2 * R * 16, R * 16, 128),
                    tc::smem_desc(v_s + ks * 2 * 128, 128, TT * 16), idesc, c > 0 || ks > 0);
      tc::commit(&sm.bar[1]);
    }
    ok = mbar_wait_bounded(&sm.bar[1], parity) && ok;
    tc::fence_after_thread_sync();
    parity ^= 1u;
  }
  if (bad_page) set_error(p.error, kErrBadPage);

  // ---- the item's partial rows: unnormalised O and (max in log2 units, sum).
  // Staged through shared memory (rows of D floats + 16 bytes: 8 consecutive
  // rows fall in 8 different 16-byte bank groups) over the operand tiles, all
  // consumed, then written row by row with whole warps on each row.
  constexpr int OP = D * 4 + 16;  // staged row pitch (bytes)
  uint8_t* o_s = sm.base;
#pragma unroll
  for (int j = 0; j < D / 8; ++j) {
    float o8[8];
    tc::ld8(tmem_o + lane_off + j * 8, o8);
    float4* dst = reinterpret_cast<float4*>(o_s + row * OP + j * 32);
    dst[0] = make_float4(o8[0], o8[1], o8[2], o8[3]);
    dst[1] = make_float4(o8[4], o8[5], o8[6], o8[7]);
  }
  const int mi = row / G;
  const int b = mi < n_mem ? sm.mem_s[mi] : -1;
  if (ok && b >= 0 && b < p.batch)
    p.part_ml[((int64_t)b * p.num_heads + kvh * G + row % G) * p.max_chunks + part] = make_float2(m_run, l_run);
  sync();
  for (int v = tid; v < R * (D / 4); v += NTH) {
    const int r = v / (D / 4), q4 = v - r * (D / 4);
    const int mr = r / G;
    const int br = mr < n_mem ? sm.mem_s[mr] : -1;
    if (ok && br >= 0 && br < p.batch) {
      const int64_t sr = ((int64_t)br * p.num_heads + kvh * G + r % G) * p.max_chunks + part;
      reinterpret_cast<float4*>(p.part_o + sr * D)[q4] = *reinterpret_cast<const float4*>(o_s + r * OP + q4 * 16);
    }
  }
  if (!ok && tid == 0) set_error(p.error, kErrTimeout);
  tc::fence_before_thread_sync();
  sync();
  tc::fence_after_thread_sync();
  return true;
}

}  // namespace ubx
