// Pre-attention step as one launch (sm_100a): per-head RMSNorm of q and k, the
// rotary embedding at each token's position, and the KV append of the rotated k
// and the raw v rows.
//
// Replaces, for the T tokens of a decode step (one per sequence) or of a prefill
// chunk, the reference's
//   xq = q_norm(xq); xk = k_norm(xk)                 engine.py:201-202 / :121-122
//   per-sequence apply_rotary_emb at pos (.item())   engine.py:204-210 / :123
//   per-token write_kv(layer, seq, pos, xk, xv)      engine.py:213-215 / :126-128
// (RMSNorm: unbox_platform/model/model.py:19-27; rotary: model.py:30-48; the
// write: kvcache.py:330-340). One warp handles one (token, head) row at a time (a
// block per token, its warps over the heads); the warps
// of K heads also store the token's K and V rows into the pool.
#include <algorithm>

#include "ubx_common.cuh"
#include "ubx_internal.h"
#include "ubx_prep.cuh"

namespace ubx {

namespace {

constexpr int kPrepWarps = 8;
constexpr int kMaxPairsPerLane = 4;  // head_dim <= 256

template <typename T>
__device__ __forceinline__ float2 load_pair(const T* p);
template <>
__device__ __forceinline__ float2 load_pair<float>(const float* p) {
  return __ldg(reinterpret_cast<const float2*>(p));
}
template <>
__device__ __forceinline__ float2 load_pair<__nv_bfloat16>(const __nv_bfloat16* p) {
  return unpack_word<__nv_bfloat16>(__ldg(reinterpret_cast<const uint32_t*>(p)));
}
template <>
__device__ __forceinline__ float2 load_pair<__half>(const __half* p) {
  return unpack_word<__half>(__ldg(reinterpret_cast<const uint32_t*>(p)));
}

template <typename T>
__device__ __forceinline__ void store_pair(T* p, float2 v);
template <>
__device__ __forceinline__ void store_pair<float>(float* p, float2 v) {
  *reinterpret_cast<float2*>(p) = v;
}
template <>
__device__ __forceinline__ void store_pair<__nv_bfloat16>(__nv_bfloat16* p, float2 v) {
  *reinterpret_cast<uint32_t*>(p) = Elem<__nv_bfloat16>::pack2(v.x, v.y);
}
template <>
__device__ __forceinline__ void store_pair<__half>(__half* p, float2 v) {
  *reinterpret_cast<uint32_t*>(p) = Elem<__half>::pack2(v.x, v.y);
}

// Raw copy of one element pair (the V row goes to the pool unchanged).
template <typename T>
__device__ __forceinline__ void copy_pair(T* dst, const T* src) {
  if constexpr (sizeof(T) == 4)
    *reinterpret_cast<uint2*>(dst) = __ldg(reinterpret_cast<const uint2*>(src));
  else
    *reinterpret_cast<uint32_t*>(dst) = __ldg(reinterpret_cast<const uint32_t*>(src));
}

template <typename T>
__global__ void __launch_bounds__(kPrepWarps * 32) qk_norm_rope_kernel(const PrepParams p) {
  const int lane = threadIdx.x & 31;
  const int rows_per_token = p.num_heads + p.num_kv_heads;
  const int np = p.head_dim / 2;
  const float inv_d = 1.f / (float)p.head_dim;
  const int64_t limit = p.num_blocks * p.block_size;
  // the page size is a power of two in practice: a shift instead of a 64-bit division
  const int bs_shift = (p.block_size & (p.block_size - 1)) == 0 ? __ffs(p.block_size) - 1 : -1;
  // a block per token (grid-stride), its warps over the token's q and k rows:
  // no division to find a row's token and head
  for (int64_t t = blockIdx.x; t < p.num_tokens; t += gridDim.x)
  for (int h = threadIdx.x >> 5; h < rows_per_token; h += kPrepWarps) {
    const bool is_q = h < p.num_heads;
    const int hk = h - p.num_heads;
    const T* x = is_q ? static_cast<const T*>(p.q_in) + t * p.q_st + (int64_t)h * p.q_sh
                      : static_cast<const T*>(p.k_in) + t * p.k_st + (int64_t)hk * p.k_sh;
    const T* w = static_cast<const T*>(is_q ? p.q_w : p.k_w);
    const int pos = __ldg(&p.positions[t]);
    const bool pos_ok = pos >= 0 && pos < p.rope_n;
    if (!pos_ok && lane == 0 && h == 0) set_error(p.error, kErrBadPosition);

    float2 v[kMaxPairsPerLane];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPairsPerLane; ++i) {
      const int j = lane + 32 * i;
      v[i] = j < np ? load_pair<T>(x + 2 * j) : make_float2(0.f, 0.f);
      ss += rounded_square<T>(v[i].x) + rounded_square<T>(v[i].y);
    }
    const float rf = rms_factor<T>(warp_sum(ss), inv_d, p.eps);

    // destinations of this row
    T* dst = nullptr;
    T* dst_cache = nullptr;
    T* dst_v = nullptr;
    const T* src_v = nullptr;
    if (is_q) {
      dst = static_cast<T*>(p.q_out) + t * p.qo_st + (int64_t)h * p.qo_sh;
    } else {
      if (p.k_out) dst = static_cast<T*>(p.k_out) + t * p.ko_st + (int64_t)hk * p.ko_sh;
      if (p.k_cache) {
        const int64_t slot = __ldg(&p.slots[t]);
        if (slot >= limit) {
          if (lane == 0 && hk == 0) set_error(p.error, kErrBadSlot);
        } else if (slot >= 0) {
          const int64_t blk = bs_shift >= 0 ? slot >> bs_shift : slot / p.block_size;
          const int64_t off = blk * p.c_sblk + (slot - blk * p.block_size) * p.c_stok + (int64_t)hk * p.c_sh;
          dst_cache = static_cast<T*>(p.k_cache) + off;
          dst_v = static_cast<T*>(p.v_cache) + off;
          src_v = static_cast<const T*>(p.v_in) + t * p.v_st + (int64_t)hk * p.v_sh;
        }
      }
    }
    const float* rope_row = p.rope + (int64_t)(pos_ok ? pos : 0) * p.rope_sp;
#pragma unroll
    for (int i = 0; i < kMaxPairsPerLane; ++i) {
      const int j = lane + 32 * i;
      if (j >= np) break;
      const float2 wv = load_pair<T>(w + 2 * j);
      const float y0 = rms_apply<T>(v[i].x, rf, wv.x), y1 = rms_apply<T>(v[i].y, rf, wv.y);
      const float2 cs = pos_ok ? __ldg(reinterpret_cast<const float2*>(rope_row) + j) : make_float2(1.f, 0.f);
      const float2 o = rotate_pair(y0, y1, cs.x, cs.y);
      const float2 out = make_float2(round_to<T>(o.x), round_to<T>(o.y));
      if (dst) store_pair<T>(dst + 2 * j, out);
      if (dst_cache) {
        store_pair<T>(dst_cache + 2 * j, out);
        copy_pair<T>(dst_v + 2 * j, src_v + 2 * j);
      }
    }
  }
}

// 16-bit rows with 16-byte-aligned rows and a head_dim that is a multiple of 8:
// each lane takes one 16-byte chunk (8 elements, 4 rotary pairs) of a row, the
// CH = head_dim / 8 lanes of a row sit in a segment of W lanes (W the power of
// two >= CH), so a warp works on 32 / W rows at once and a row's sum of squares
// is a W-lane butterfly. The launch's (token, head) rows are taken 16 per block
// pass (8 warps x 2 rows) by a persistent grid, so every SM gets the same number
// of passes within one; every load of a row (x, weight, rotary pairs, the V row)
// is issued before the sum is reduced. Same rounding points as
// qk_norm_rope_kernel.
// Five blocks per SM (48 registers, no spills): more warps to hide each row's
// memory round trip than the four that 64 registers allow.
constexpr int kVecBlocksPerSm = 5;

template <typename T, int W>
__global__ void __launch_bounds__(kPrepWarps * 32, kVecBlocksPerSm) qk_norm_rope_vec_kernel(const PrepParams p) {
  constexpr int RPW = 32 / W;  // rows of one warp at a time
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int seg = lane / W, c = lane % W;
  const int CH = p.head_dim / 8;
  const int rows_per_token = p.num_heads + p.num_kv_heads;
  const float inv_d = 1.f / (float)p.head_dim;
  const int64_t limit = p.num_blocks * p.block_size;
  const int bs_shift = (p.block_size & (p.block_size - 1)) == 0 ? __ffs(p.block_size) - 1 : -1;
  // every (token, head) row of the launch, 16 rows per block pass, grid-stride
  const int64_t total_rows = p.num_tokens * rows_per_token;
  const int rows_per_pass = nwarps * RPW;
  for (int64_t base = (int64_t)blockIdx.x * rows_per_pass; base < total_rows;
       base += (int64_t)gridDim.x * rows_per_pass) {
    const int64_t R = base + warp * RPW + seg;
    const int64_t t = R / rows_per_token;
    const int h = (int)(R - t * rows_per_token);
    const bool live = c < CH && R < total_rows;  // segment-uniform
    const int pos = live ? __ldg(&p.positions[t]) : 0;
    const bool pos_ok = pos >= 0 && pos < p.rope_n;
    if (live && !pos_ok && c == 0 && h == 0) set_error(p.error, kErrBadPosition);
    const int64_t slot = (live && p.k_cache) ? __ldg(&p.slots[t]) : -1;
    const float4* rope_row = reinterpret_cast<const float4*>(p.rope + (int64_t)(pos_ok ? pos : 0) * p.rope_sp);
    const bool is_q = h < p.num_heads;
    const int hk = h - p.num_heads;
    const bool to_cache = !is_q && slot >= 0 && slot < limit;
    uint32_t xw[4] = {0u, 0u, 0u, 0u}, ww[4] = {0u, 0u, 0u, 0u};  // element pairs of x and of the weight
    float4 cs[2] = {make_float4(1.f, 0.f, 1.f, 0.f), make_float4(1.f, 0.f, 1.f, 0.f)};
    uint4 vrow = make_uint4(0, 0, 0, 0);
    float ss = 0.f;
    if (live) {
      const T* src = is_q ? static_cast<const T*>(p.q_in) + t * p.q_st + (int64_t)h * p.q_sh
                          : static_cast<const T*>(p.k_in) + t * p.k_st + (int64_t)hk * p.k_sh;
      const uint4 xr = __ldg(reinterpret_cast<const uint4*>(src) + c);
      const uint4 wr = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(is_q ? p.q_w : p.k_w)) + c);
      if (pos_ok) {
        cs[0] = __ldg(rope_row + 2 * c);
        cs[1] = __ldg(rope_row + 2 * c + 1);
      }
      if (to_cache)
        vrow = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(p.v_in) + t * p.v_st +
                                                    (int64_t)hk * p.v_sh) + c);
      xw[0] = xr.x, xw[1] = xr.y, xw[2] = xr.z, xw[3] = xr.w;
      ww[0] = wr.x, ww[1] = wr.y, ww[2] = wr.z, ww[3] = wr.w;
#pragma unroll
      for (int i = 0; i < 4; ++i) {  // rounded squares (packed), summed in element order
        const float2 sq = unpack_word<T>(mul2_rn<T>(xw[i], xw[i]));
        ss += sq.x;
        ss += sq.y;
      }
    }
#pragma unroll
    for (int off = W / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (!live) continue;
    const float rf = rms_factor<T>(ss, inv_d, p.eps);  // a dtype value
    const uint32_t rf2 = Elem<T>::pack2(rf, rf);
    // (x * r) * w with each product rounded (packed multiplies: the values of
    // rms_apply), the rotation in fp32, and the output rounded by the packing
    uint32_t ow[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 y = unpack_word<T>(mul2_rn<T>(mul2_rn<T>(xw[i], rf2), ww[i]));
      const float4& c4 = cs[i >> 1];
      const float2 o = rotate_pair(y.x, y.y, (i & 1) ? c4.z : c4.x, (i & 1) ? c4.w : c4.y);
      ow[i] = Elem<T>::pack2(o.x, o.y);
    }
    const uint4 packed = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    if (is_q) {
      reinterpret_cast<uint4*>(static_cast<T*>(p.q_out) + t * p.qo_st + (int64_t)h * p.qo_sh)[c] = packed;
      continue;
    }
    if (p.k_out) reinterpret_cast<uint4*>(static_cast<T*>(p.k_out) + t * p.ko_st + (int64_t)hk * p.ko_sh)[c] = packed;
    if (p.k_cache && slot >= limit && c == 0 && hk == 0) set_error(p.error, kErrBadSlot);
    if (to_cache) {
      const int64_t blk = bs_shift >= 0 ? slot >> bs_shift : slot / p.block_size;
      const int64_t off = blk * p.c_sblk + (slot - blk * p.block_size) * p.c_stok + (int64_t)hk * p.c_sh;
      reinterpret_cast<uint4*>(static_cast<T*>(p.k_cache) + off)[c] = packed;
      reinterpret_cast<uint4*>(static_cast<T*>(p.v_cache) + off)[c] = vrow;
    }
  }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// SMs of the current device (looked up once per device; 148 if the query fails).
int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// Rows, strides, weights and rotary rows on 16-byte boundaries, head_dim a
// multiple of 8 (at most 256): the 16-byte-per-lane kernel applies.
bool vec_ok(const PrepParams& p) {
  const auto m8 = [](int64_t s) { return (s & 7) == 0; };  // element strides of 16-bit rows
  bool ok = p.head_dim % 8 == 0 && p.head_dim <= 256 && aligned16(p.q_in) && aligned16(p.k_in) &&
            aligned16(p.q_out) && aligned16(p.q_w) && aligned16(p.k_w) && aligned16(p.rope) &&
            (p.rope_sp & 3) == 0 && m8(p.q_st) && m8(p.q_sh) && m8(p.k_st) && m8(p.k_sh) && m8(p.qo_st) &&
            m8(p.qo_sh);
  if (p.k_out) ok = ok && aligned16(p.k_out) && m8(p.ko_st) && m8(p.ko_sh);
  if (p.k_cache)
    ok = ok && aligned16(p.k_cache) && aligned16(p.v_cache) && aligned16(p.v_in) && m8(p.c_sblk) && m8(p.c_stok) &&
         m8(p.c_sh) && m8(p.v_st) && m8(p.v_sh);
  return ok;
}

template <typename T>
cudaError_t launch_vec(const PrepParams& p, int blocks, cudaStream_t stream) {
  const int ch = p.head_dim / 8;
  const int w = ch <= 8 ? 8 : ch <= 16 ? 16 : 32;
  const dim3 block(kPrepWarps * 32);
  if (w == 8) qk_norm_rope_vec_kernel<T, 8><<<blocks, block, 0, stream>>>(p);
  else if (w == 16) qk_norm_rope_vec_kernel<T, 16><<<blocks, block, 0, stream>>>(p);
  else qk_norm_rope_vec_kernel<T, 32><<<blocks, block, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_qk_norm_rope(int dtype, const PrepParams& p, cudaStream_t stream) {
  if (p.num_tokens == 0) return cudaSuccess;
  const int blocks = (int)(p.num_tokens < 148 * 32 ? p.num_tokens : 148 * 32);  // a block per token
  if (dtype != 0 && vec_ok(p)) {
    // a persistent grid of kVecBlocksPerSm blocks per SM over every row, 16 at a time
    const int64_t vb = (p.num_tokens * (p.num_heads + p.num_kv_heads) + 15) / 16;
    const int64_t cap = (int64_t)kVecBlocksPerSm * num_sms();
    const int vblocks = (int)(vb < cap ? vb : cap);
    return dtype == 1 ? launch_vec<__nv_bfloat16>(p, vblocks, stream) : launch_vec<__half>(p, vblocks, stream);
  }
  switch (dtype) {
    case 0: qk_norm_rope_kernel<float><<<blocks, kPrepWarps * 32, 0, stream>>>(p); break;
    case 1: qk_norm_rope_kernel<__nv_bfloat16><<<blocks, kPrepWarps * 32, 0, stream>>>(p); break;
    case 2: qk_norm_rope_kernel<__half><<<blocks, kPrepWarps * 32, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace ubx
