// Allocation-free variant of the paged decode-attention entry point.
//
// Some callers cannot allocate device memory for a workspace: an engine that
// hands all free HBM to its own KV-cache pool at start-up and owns every later
// allocation, or a binding from another language that only has the input and
// output buffers and no handle on a device allocator. For them this file keeps
// the attention kernel's scratch (merge counters and the partial results of
// sequences split across CTAs) in a fixed array in the library's own device
// memory instead of a caller workspace.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds kNoAllocScratchBytes of it until the process exits. Its name in
// host code is only a stand-in for the symbol, never a device address, so the
// address is looked up once per device with cudaGetSymbolAddress (with that
// device current) and cached; the first call on each device performs that
// lookup, so make the first call on a device before any stream capture. The
// cache is keyed by device ordinal for the life of the process: it assumes the
// device's primary context, so cudaDeviceReset (which unloads the module) and
// calls made under another driver-API context of the same device are not
// supported.
#include <cstdio>
#include <mutex>
#include <string>

#include "ubx_internal.h"
#include "../../include/unbox_b200.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per GPU
static_assert(kNoAllocScratchBytes > ubx::kWsZeroBytes, "scratch holds the fixed prefix");

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};

int cuda_status(cudaError_t e, const char* what) {
  std::string m = std::string("ubx_paged_decode_attention_noalloc: ") + what + ": " + cudaGetErrorString(e);
  ubx::set_last_error(m.c_str());
  return UBX_ERR_CUDA;
}

// Device address of g_decode_scratch on the current device (looked up once per device).
cudaError_t scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

int ubx_paged_decode_attention_noalloc(const void* q, int64_t q_s_b, int64_t q_s_h, const void* k_cache,
                                       const void* v_cache, int64_t c_s_block, int64_t c_s_tok, int64_t c_s_head,
                                       const int32_t* block_table, int64_t bt_s_row, const int32_t* context_lens,
                                       void* out, int64_t o_s_b, int64_t o_s_h, int batch, int num_heads,
                                       int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                                       int max_blocks_per_seq, float scale, int dtype, int schedule, int split_pages,
                                       int32_t* error_word, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return cuda_status(e, "scratch address lookup (cudaGetSymbolAddress)");
  // The array keeps whatever the previous call left: the error word and the
  // counters (the whole zero-initialised prefix of the workspace) are re-zeroed
  // on `stream` once the arguments have passed every check, just before the
  // launch; a rejected call leaves the array untouched.
  int st = ubx::paged_decode_attention_cleared(q, q_s_b, q_s_h, k_cache, v_cache, c_s_block, c_s_tok, c_s_head,
                                               block_table, bt_s_row, context_lens, out, o_s_b, o_s_h, batch,
                                               num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                                               max_blocks_per_seq, scale, dtype, schedule, split_pages, scratch,
                                               kNoAllocScratchBytes, ubx::kWsZeroBytes, stream);
  if (st == UBX_ERR_WORKSPACE) {
    // the only workspace here is the fixed array: say so, with its limit
    char msg[512];
    snprintf(msg, sizeof(msg),
             "ubx_paged_decode_attention_noalloc: these sizes need more scratch than the fixed %zu-byte "
             "array holds (%s); call ubx_paged_decode_attention with a caller workspace instead",
             kNoAllocScratchBytes, ubx::last_error());
    ubx::set_last_error(msg);
    return st;
  }
  if (st != UBX_OK || batch <= 0) return st;
  if (error_word) {
    e = cudaMemcpyAsync(error_word, scratch, sizeof(int32_t), cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_status(e, "error word copy");
  }
  return UBX_OK;
}

}  // extern "C"
