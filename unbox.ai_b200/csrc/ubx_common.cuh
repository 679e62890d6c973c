// Device helpers shared by the unbox_b200 kernels (sm_100a).
//
// mbarrier + bulk-copy (cp.async.bulk, TMA engine) primitives written as inline PTX, the
// 16-byte element converters used when K/V chunks are unpacked from shared
// memory, and the device error word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/unbox_b200.h"

namespace ubx {

// Bits of the device error word (one int32 in the workspace). Kernels never trap:
// they record the condition here and skip the offending access; the host reads
// the word back with ubx_read_device_error().
enum : int32_t {
  kErrBadPage = UBX_DEVERR_BAD_PAGE,          // page id outside [0, num_blocks)
  kErrCtxTooLong = UBX_DEVERR_CTX_TOO_LONG,   // context needs more pages than the table row
  kErrNegCtx = UBX_DEVERR_NEG_CTX,            // negative context length
  kErrTimeout = UBX_DEVERR_TIMEOUT,           // a pipeline wait exceeded its bound
  kErrBadSlot = UBX_DEVERR_BAD_SLOT,          // append slot >= num_blocks * block_size
  kErrBadPosition = UBX_DEVERR_BAD_POSITION,  // rotary position outside the table
  kErrBadWork = UBX_DEVERR_BAD_WORK,          // a cascade work or merge item out of range
};

__device__ __forceinline__ void set_error(int32_t* err, int32_t bit) {
  if (err) atomicOr(err, bit);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- programmatic dependent launch
// Lets the next kernel on the stream launch once every CTA of this grid got here.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Waits until the grids this one depends on have completed and their memory is
// visible (returns at once when the launch had no programmatic dependency).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete, for at most ~2^31 SM
// clocks (about a second). Returns false on timeout; the caller records
// kErrTimeout and unwinds instead of spinning forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > (1ll << 31)) return false;
  }
  return true;
}

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Same for global memory: generic writes before a later TMA read of them.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
// Bulk copy (TMA engine, non-tensor) of `bytes` contiguous bytes global ->
// shared, completion counted in bytes on `bar`. Both addresses 16-byte
// aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_copy_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Atomic add with acquire-release semantics at GPU scope: the writes that
// precede it (in this thread, or in threads ordered before it by a barrier)
// are visible to whoever observes the new value, and whatever this thread does
// after it sees the writes that preceded the values it observed. One round trip
// in place of a fence and an atomic.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int32_t* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Relaxed store at GPU scope (no ordering, no round trip to wait for).
__device__ __forceinline__ void st_relaxed_gpu(int32_t* p, int v) {
  asm volatile("st.relaxed.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// L2 eviction policy for data read once per launch (KV pages streamed from
// HBM): the lines it fills are evicted first, so the small data every launch
// re-reads (block tables, context lengths, queries, partial results) stays in L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// bulk_copy_g2s with an L2 cache policy (l2_policy_evict_first) for the source lines.
__device__ __forceinline__ void bulk_copy_g2s_hint(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                                   uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(smem_u32(bar)),
        "l"(policy)
      : "memory");
}

// Tiled tensor copy global -> shared (TMA engine) of the box at coordinates
// (c0, c1, c2) of a 3-D tensor map, completing `bytes` on the mbarrier. The map
// lives in kernel parameter space (a __grid_constant__ argument). c0 times the
// element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
        "r"(smem_u32(bar))
      : "memory");
}

// Asks L2 to fetch `bytes` of global memory (TMA engine, no shared memory, no
// completion to wait for). Address 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* gmem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes)
               : "memory");
}

// Bulk copy shared -> global (TMA engine, non-tensor), tracked in the issuing
// thread's bulk async-groups. Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_s2g(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               ::"l"(reinterpret_cast<uint64_t>(gmem_dst)), "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}

// Closes the bulk operations issued so far into one group (an empty group if none).
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Until at most N of this thread's most recent bulk groups still read their source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Until at most N of this thread's most recent bulk groups are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// 16-byte global -> shared copy without register staging (cp.async, L2 only);
// both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
               ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(gmem_src))
               : "memory");
}

// Closes this thread's cp.async copies into a group and waits until all are done.
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Explicit shared-memory accesses (ld/st.shared rather than generic addressing).
__device__ __forceinline__ int4 lds_int4(const void* p) {
  int4 v;
  asm volatile("ld.shared.v4.s32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void sts_int4(void* p, int4 v) {
  asm volatile("st.shared.v4.s32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ int lds_int(const void* p) {
  int v;
  asm volatile("ld.shared.s32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}

// ---------------------------------------------------------------- elements
template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static constexpr int kPerChunk = 4;   // elements per 16-byte chunk
  __device__ __forceinline__ static void unpack(const uint4& v, float (&f)[4]) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[4]) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
  __device__ __forceinline__ static float to_float(float x) { return x; }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kPerChunk = 8;
  // bf16 is the upper half of an fp32: widening is a shift or a mask.
  __device__ __forceinline__ static void unpack(const uint4& v, float (&f)[8]) {
    f[0] = __uint_as_float(v.x << 16);
    f[1] = __uint_as_float(v.x & 0xffff0000u);
    f[2] = __uint_as_float(v.y << 16);
    f[3] = __uint_as_float(v.y & 0xffff0000u);
    f[4] = __uint_as_float(v.z << 16);
    f[5] = __uint_as_float(v.z & 0xffff0000u);
    f[6] = __uint_as_float(v.w << 16);
    f[7] = __uint_as_float(v.w & 0xffff0000u);
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[8]) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
  }
  __device__ __forceinline__ static float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
};

template <>
struct Elem<__half> {
  static constexpr int kPerChunk = 8;
  __device__ __forceinline__ static void unpack(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 p = __half22float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
  __device__ __forceinline__ static uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[8]) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
  }
  __device__ __forceinline__ static float to_float(__half x) { return __half2float(x); }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace ubx
