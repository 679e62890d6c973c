// Tensor-core helpers shared by the decode and cascade kernels (sm_100a):
// ldmatrix loads and the m16n8k16 mma.sync with 16-bit inputs, fp32 accumulate.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "ubx_common.cuh"

namespace ubx {

// ldmatrix: four 8x8 b16 matrices, row addresses supplied by lanes 8i..8i+7.
__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_trans(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

// D(16x8, f32) += A(16x16) * B(16x8) (A row-major, B column-major, 16-bit
// inputs) for an A whose rows 8..15 are zero (the padding rows of a q-head
// tile): only D rows 0..7 are kept (d[0], d[1] of this lane); rows 8..15 come
// back as zeros into registers that die at once, so they hold no accumulator.
template <typename T>
__device__ __forceinline__ void mma16816_top(float (&d)[2], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  float dead0, dead1;
  const float zero = 0.f;
  if constexpr (sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %10, %10};"
        : "+f"(d[0]), "+f"(d[1]), "=f"(dead0), "=f"(dead1)
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1), "f"(zero));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %10, %10};"
        : "+f"(d[0]), "+f"(d[1]), "=f"(dead0), "=f"(dead1)
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1), "f"(zero));
  }
  (void)dead0;
  (void)dead1;
}

// D(16x8, f32) += A(16x16) * B(16x8), A row-major (a0: rows 0-7 / k 0-7, a1: rows
// 8-15 / k 0-7, a2: rows 0-7 / k 8-15, a3: rows 8-15 / k 8-15), B column-major.
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

}  // namespace ubx
