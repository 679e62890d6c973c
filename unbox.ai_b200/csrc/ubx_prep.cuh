// Device helpers of the pre-attention step: per-head RMSNorm of q and k followed
// by the rotary embedding, with the rounding of the reference's tensor ops.
//
// The reference computes, per head row x of length D in the model dtype
// (unbox_platform/model/model.py:25-27 RMSNorm.forward, then :36-48
// apply_rotary_emb; the engine calls them at engine.py:201-210 for a decode step
// and :121-123 for a prefill chunk):
//   s   = x.pow(2)                  -> rounded to the dtype, element by element
//   m   = s.mean(-1)                -> fp32 sum * (1/D), rounded
//   r   = rsqrt(m + eps)            -> m + eps rounded, rsqrt rounded
//   y   = (x * r) * weight          -> each product rounded
//   out = (y0 + i y1) * (cos + i sin) per pair (2j, 2j+1), in fp32, rounded
// For 16-bit tensors every tensor op above rounds its fp32 result to the dtype;
// the helpers below round at the same points so the kernels produce the values
// the reference's tensor ops produce (fp32 tensors: no rounding).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace ubx {

template <typename T>
__device__ __forceinline__ float round_to(float x);
template <>
__device__ __forceinline__ float round_to<float>(float x) { return x; }
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
template <>
__device__ __forceinline__ float round_to<__half>(float x) { return __half2float(__float2half_rn(x)); }

// Product of two element pairs of a 16-bit row (one 32-bit word each), rounded
// to the dtype by one packed multiply. The exact product of two bf16 (or two
// fp16) values fits an fp32 significand, so this equals the fp32 product
// rounded to the dtype, element by element: the value of round_to(a * b).
// The one exception is a product below the smallest normal fp32 (2^-126; for a
// square, |x| below 2^-63): the fp32 path then rounds twice and the last bit
// may differ.
template <typename T>
__device__ __forceinline__ uint32_t mul2_rn(uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ uint32_t mul2_rn<__nv_bfloat16>(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162*>(&a), *reinterpret_cast<const __nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
template <>
__device__ __forceinline__ uint32_t mul2_rn<__half>(uint32_t a, uint32_t b) {
  __half2 r = __hmul2_rn(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// x.pow(2) of one element (the product is not fused into the running sum)
template <typename T>
__device__ __forceinline__ float rounded_square(float x) { return round_to<T>(__fmul_rn(x, x)); }

// rsqrt(mean + eps) from the row's sum of rounded squares
template <typename T>
__device__ __forceinline__ float rms_factor(float sum_sq, float inv_d, float eps) {
  const float mean = round_to<T>(__fmul_rn(sum_sq, inv_d));
  const float ms = round_to<T>(__fadd_rn(mean, eps));
  return round_to<T>(rsqrtf(ms));
}

// (x * r) * w
template <typename T>
__device__ __forceinline__ float rms_apply(float x, float r, float w) {
  return round_to<T>(__fmul_rn(round_to<T>(__fmul_rn(x, r)), w));
}

// complex product (a + ib)(c + is) as torch's complex64 multiply: ac - bs, as + bc
__device__ __forceinline__ float2 rotate_pair(float a, float b, float c, float s) {
  return make_float2(__fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)), __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c)));
}

// Two consecutive elements of a 16-bit row as floats (one 32-bit word).
template <typename T>
__device__ __forceinline__ float2 unpack_word(uint32_t w);
template <>
__device__ __forceinline__ float2 unpack_word<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 unpack_word<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

}  // namespace ubx
