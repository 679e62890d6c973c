// C ABI of the KV hand-off: wire header, page copy, peer access and CUDA IPC
// (declared in include/unbox_b200.h; the kernel is in kv_transfer.cu).
#include <cuda.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "ubx_internal.h"
#include "../../include/unbox_b200.h"

namespace {

int hfail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int hfail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  ubx::set_last_error(buf);
  return status;
}

int hcuda(cudaError_t e, const char* what) { return hfail(UBX_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e)); }

int elem_bytes(int dtype) { return dtype == UBX_DTYPE_F32 ? 4 : 2; }

bool valid_dtype(int dtype) { return dtype == UBX_DTYPE_F32 || dtype == UBX_DTYPE_BF16 || dtype == UBX_DTYPE_F16; }

uint64_t payload_size(int dtype, uint64_t layers, uint64_t kvh, uint64_t d, uint64_t bs, uint64_t pages) {
  return layers * 2 * pages * bs * kvh * d * (uint64_t)elem_bytes(dtype);
}

static_assert(sizeof(ubx_kv_wire_header) == 64, "wire header is 64 bytes");

}  // namespace

extern "C" {

int ubx_kv_wire_header_init(ubx_kv_wire_header* h, int dtype, int num_layers, int num_kv_heads, int head_dim,
                            int block_size, int num_pages, uint64_t checksum) {
  ubx::set_last_error("");
  if (!h) return hfail(UBX_ERR_INVALID_ARGUMENT, "null header");
  if (!valid_dtype(dtype)) return hfail(UBX_ERR_INVALID_ARGUMENT, "unknown dtype code %d", dtype);
  if (num_layers <= 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_pages < 0)
    return hfail(UBX_ERR_INVALID_ARGUMENT, "bad geometry");
  memset(h, 0, sizeof(*h));
  memcpy(h->magic, UBX_KV_WIRE_MAGIC, 8);
  h->version = UBX_KV_WIRE_VERSION;
  h->header_bytes = sizeof(*h);
  h->dtype = (uint32_t)dtype;
  h->num_layers = (uint32_t)num_layers;
  h->num_kv_heads = (uint32_t)num_kv_heads;
  h->head_dim = (uint32_t)head_dim;
  h->block_size = (uint32_t)block_size;
  h->num_pages = (uint32_t)num_pages;
  h->payload_bytes = payload_size(dtype, num_layers, num_kv_heads, head_dim, block_size, num_pages);
  h->checksum = checksum;
  return UBX_OK;
}

int ubx_kv_wire_header_check(const ubx_kv_wire_header* h, int dtype, int num_layers, int num_kv_heads, int head_dim,
                             int block_size, uint64_t payload_bytes) {
  ubx::set_last_error("");
  if (!h) return hfail(UBX_ERR_INVALID_ARGUMENT, "null header");
  if (memcmp(h->magic, UBX_KV_WIRE_MAGIC, 8) != 0) return hfail(UBX_ERR_INVALID_ARGUMENT, "not a KV page message");
  if (h->version != UBX_KV_WIRE_VERSION || h->header_bytes != sizeof(*h))
    return hfail(UBX_ERR_INVALID_ARGUMENT, "wire version %u / header of %u bytes not understood", h->version,
                 h->header_bytes);
  if (!valid_dtype((int)h->dtype)) return hfail(UBX_ERR_INVALID_ARGUMENT, "unknown payload dtype %u", h->dtype);
  if ((int)h->dtype != dtype)
    return hfail(UBX_ERR_UNSUPPORTED, "payload dtype %u differs from the pool's %d (no conversion)", h->dtype, dtype);
  if ((int)h->num_layers != num_layers || (int)h->num_kv_heads != num_kv_heads || (int)h->head_dim != head_dim ||
      (int)h->block_size != block_size)
    return hfail(UBX_ERR_UNSUPPORTED, "payload geometry (L=%u, KVH=%u, D=%u, bs=%u) differs from the pool's "
                                      "(L=%d, KVH=%d, D=%d, bs=%d)",
                 h->num_layers, h->num_kv_heads, h->head_dim, h->block_size, num_layers, num_kv_heads, head_dim,
                 block_size);
  const uint64_t want = payload_size(dtype, num_layers, num_kv_heads, head_dim, block_size, h->num_pages);
  if (h->payload_bytes != want || payload_bytes != want)
    return hfail(UBX_ERR_INVALID_ARGUMENT, "payload of %llu bytes (header says %llu), %u pages need %llu",
                 (unsigned long long)payload_bytes, (unsigned long long)h->payload_bytes, h->num_pages,
                 (unsigned long long)want);
  return UBX_OK;
}

int ubx_kv_pages_copy(const void* src, int64_t src_s_layer, int64_t src_s_kv, int64_t src_s_block,
                      const int32_t* src_pages, int64_t src_num_blocks, void* dst, int64_t dst_s_layer,
                      int64_t dst_s_kv, int64_t dst_s_block, const int32_t* dst_pages, int64_t dst_num_blocks,
                      int num_layers, int num_pages, int64_t page_elems, int dtype, uint64_t* checksum,
                      int32_t* error_word, void* stream) {
  ubx::set_last_error("");
  if (!valid_dtype(dtype)) return hfail(UBX_ERR_INVALID_ARGUMENT, "unknown dtype code %d", dtype);
  if (num_layers <= 0 || num_pages < 0 || page_elems <= 0) return hfail(UBX_ERR_INVALID_ARGUMENT, "bad geometry");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (checksum) {
    cudaError_t e = cudaMemsetAsync(checksum, 0, sizeof(uint64_t), s);
    if (e != cudaSuccess) return hcuda(e, "checksum memset");
  }
  if (num_pages == 0) return UBX_OK;
  if (!src || !dst) return hfail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  if ((src_pages && src_num_blocks <= 0) || (dst_pages && dst_num_blocks <= 0))
    return hfail(UBX_ERR_INVALID_ARGUMENT, "a pool side needs its num_blocks");
  const int64_t es = elem_bytes(dtype);
  const int64_t pb = page_elems * es;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  auto m16 = [&](int64_t st) { return ((st * es) & 15) == 0; };
  if (!a16(src) || !a16(dst) || (pb & 15) || !m16(src_s_layer) || !m16(src_s_kv) || !m16(src_s_block) ||
      !m16(dst_s_layer) || !m16(dst_s_kv) || !m16(dst_s_block))
    return hfail(UBX_ERR_INVALID_ARGUMENT, "page bases, strides and page size must be multiples of 16 bytes");
  if ((!src_pages && (src_s_block != page_elems || src_s_kv != (int64_t)num_pages * page_elems ||
                      src_s_layer != 2 * (int64_t)num_pages * page_elems)) ||
      (!dst_pages && (dst_s_block != page_elems || dst_s_kv != (int64_t)num_pages * page_elems ||
                      dst_s_layer != 2 * (int64_t)num_pages * page_elems)))
    return hfail(UBX_ERR_INVALID_ARGUMENT, "a packed side must have the wire payload's strides");
  if ((int64_t)num_layers * 2 * num_pages * (pb / 16) >= ((int64_t)1 << 31))
    return hfail(UBX_ERR_UNSUPPORTED, "one call copies less than 32 GiB; split the pages over several calls");
  ubx::KvCopyParams p;
  p.src = src;
  p.src_s_layer = src_s_layer * es;
  p.src_s_kv = src_s_kv * es;
  p.src_s_block = src_s_block * es;
  p.src_pages = src_pages;
  p.src_num_blocks = src_num_blocks;
  p.dst = dst;
  p.dst_s_layer = dst_s_layer * es;
  p.dst_s_kv = dst_s_kv * es;
  p.dst_s_block = dst_s_block * es;
  p.dst_pages = dst_pages;
  p.dst_num_blocks = dst_num_blocks;
  p.num_layers = num_layers;
  p.num_pages = num_pages;
  p.page_bytes = pb;
  p.checksum = reinterpret_cast<unsigned long long*>(checksum);
  p.error = error_word;
  {
    // copies between two buffers of this GPU take the TMA bulk path; when
    // either side is another GPU's memory (peer access, IPC mapping) the copy
    // runs as plain 16-byte loads and stores: a peer destination never gets a
    // TMA store, a peer source (a decode worker pulling pages) never a TMA load
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return hcuda(e, "cudaGetDevice");
    auto on_this_gpu = [&](const void* ptr) {
      cudaPointerAttributes a;
      cudaError_t pe = cudaPointerGetAttributes(&a, ptr);
      if (pe != cudaSuccess) cudaGetLastError();
      return pe == cudaSuccess && a.type == cudaMemoryTypeDevice && a.device == dev;
    };
    p.cross_gpu = !on_this_gpu(dst) || !on_this_gpu(src);
  }
  cudaError_t e = ubx::launch_kv_pages_copy(p, s);
  if (e != cudaSuccess) return hcuda(e, "kv_pages_copy launch");
  return UBX_OK;
}

int ubx_enable_peer_access(int peer_device) {
  ubx::set_last_error("");
  int dev = 0, can = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return hcuda(e, "cudaGetDevice");
  if (peer_device == dev) return UBX_OK;
  e = cudaDeviceCanAccessPeer(&can, dev, peer_device);
  if (e != cudaSuccess) return hcuda(e, "cudaDeviceCanAccessPeer");
  if (!can) return hfail(UBX_ERR_UNSUPPORTED, "device %d cannot access device %d", dev, peer_device);
  e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();  // the call leaves its status as the last error: clear it
    return UBX_OK;
  }
  if (e != cudaSuccess) return hcuda(e, "cudaDeviceEnablePeerAccess");
  return UBX_OK;
}

int ubx_ipc_get_handle(const void* dev_ptr, void* handle_out, uint64_t* offset_out) {
  ubx::set_last_error("");
  if (!dev_ptr || !handle_out || !offset_out) return hfail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  // the allocation's base: a driver call, reached through the runtime so that the
  // library does not link the driver library directly
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return hfail(UBX_ERR_CUDA, "cuMemGetAddressRange not available");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = reinterpret_cast<GetRange>(fn)(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr));
  if (r != CUDA_SUCCESS) return hfail(UBX_ERR_CUDA, "cuMemGetAddressRange failed (%d)", (int)r);
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return hcuda(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (uint64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return UBX_OK;
}

int ubx_ipc_open_handle(const void* handle, void** base_out) {
  ubx::set_last_error("");
  if (!handle || !base_out) return hfail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return hcuda(e, "cudaIpcOpenMemHandle");
  return UBX_OK;
}

int ubx_ipc_close_handle(void* base) {
  ubx::set_last_error("");
  if (!base) return hfail(UBX_ERR_INVALID_ARGUMENT, "null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return hcuda(e, "cudaIpcCloseMemHandle");
  return UBX_OK;
}

}  // extern "C"
