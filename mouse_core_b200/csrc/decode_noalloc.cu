// Decode attention for callers that cannot allocate device memory.
//
// mb_decode_attention needs a caller-provided workspace (the split-KV work
// list, per-chunk partial results and merge counters). Some callers have no
// way to provide one: an FFI caller (ctypes, cgo, JNI) that only holds the
// pointers its framework handed it and has no device allocator to call, or a
// process whose device memory belongs to another framework's caching
// allocator, where an extra cudaMalloc would bypass that allocator's
// accounting and limits. mb_decode_attention_noalloc serves them from a
// fixed scratch array compiled into this library instead.
//
// The scratch is a file-scope __device__ array of MB_NOALLOC_SCRATCH_BYTES.
// Every GPU that loads the library holds it until the process exits. Host
// code cannot pass the array's name to a kernel (on the host the name is only
// a stand-in for the device symbol), so the first call on each device looks
// up the array's device address with cudaGetSymbolAddress while that device is
// current and caches it; make that first call before capturing any stream.
#include <mutex>

#include "../../include/mouse_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace mb {
static __device__ __align__(256) uint8_t g_noalloc_scratch[MB_NOALLOC_SCRATCH_BYTES];
}  // namespace mb

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
uint8_t* g_noalloc_base[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once
// per device, with that device current). The kernels run on `stream`, so the
// stream must belong to that same device: the address is only valid there.
int noalloc_scratch_address(cudaStream_t stream, uint8_t** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(MB_ERR_UNSUPPORTED, "device ordinal out of range");
  int stream_dev = -1;
  e = cudaStreamGetDevice(stream, &stream_dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamGetDevice");
  if (stream_dev != dev)
    return fail(MB_ERR_INVALID_ARG, "the stream belongs to device " + std::to_string(stream_dev) +
                                        " but device " + std::to_string(dev) +
                                        " is current; make the stream's device current first");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_base[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, mb::g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
    g_noalloc_base[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_noalloc_base[dev];
  return MB_OK;
}

}  // namespace

extern "C" int mb_decode_attention_noalloc(const void* q, const void* k_pool, const void* v_pool, int num_pages,
                                           const int32_t* block_table, int max_pages, const int32_t* q_pos,
                                           const int32_t* kv_len, int batch, int q_len, int q_heads, int kv_heads,
                                           int head_dim, int page_size, float scale, int max_kv_len, void* out,
                                           mb_stream_t stream) {
  int rc = check_decode_shape(batch, q_len, q_heads, kv_heads, head_dim, page_size);
  if (rc) return rc;
  if (batch == 0 || q_len == 0) return MB_OK;
  const int rows = (q_heads / kv_heads) * q_len;
  const size_t need = mb_decode_workspace_bytes(batch, kv_heads, rows, head_dim, max_kv_len);
  if (need > (size_t)MB_NOALLOC_SCRATCH_BYTES)
    return fail(MB_ERR_WORKSPACE, "this shape needs " + std::to_string(need) +
                                      " bytes of scratch, more than the built-in MB_NOALLOC_SCRATCH_BYTES (" +
                                      std::to_string((size_t)MB_NOALLOC_SCRATCH_BYTES) +
                                      "); use mb_decode_attention with a caller-provided workspace");
  uint8_t* scratch = nullptr;
  if ((rc = noalloc_scratch_address((cudaStream_t)stream, &scratch))) return rc;
  // plan_ready = 0: the work list is rebuilt and the merge counters cleared on
  // every call, so nothing depends on what the previous call left behind.
  return mb_decode_attention(q, k_pool, v_pool, num_pages, block_table, max_pages, q_pos, kv_len, batch, q_len,
                             q_heads, kv_heads, head_dim, page_size, scale, max_kv_len, /*plan_ready=*/0, out,
                             scratch, (size_t)MB_NOALLOC_SCRATCH_BYTES, stream);
}
