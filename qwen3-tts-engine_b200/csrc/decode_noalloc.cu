// Paged decode attention for callers that cannot allocate device memory.
//
// q3_paged_decode needs a caller-provided workspace (split-K partials and ticket counters). Some callers cannot
// provide one: code that runs where a cudaMalloc is not allowed or not wanted -- a host runtime whose device memory is
// owned by a fixed arena it does not control, a plugin whose host framework forbids allocation in the call, or code
// that must not allocate on a latency-critical path. q3_paged_decode_noalloc serves them from a fixed scratch array
// compiled into this library instead: nothing is allocated, ever.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes (16 MiB) that every GPU loading this library
// keeps until the process exits. Host code cannot use the array's name as a device address, so the first call on each
// device (with that device current) asks the runtime for the address with cudaGetSymbolAddress and caches it; make
// that first call before any stream capture. The cached address belongs to the device's current context: after a
// cudaDeviceReset on that device the library must be reloaded (the cache would point into the destroyed context).
// All calls on a device share the array and it keeps the last call's contents: every accepted call clears the ticket
// counters it will use (an asynchronous memset on the call's stream, queued only after all argument checks passed, so
// a refused call touches nothing), and calls that overlap on the GPU -- different streams, or different host threads --
// race on the array.
#include <cuda_runtime.h>

#include "q3_common.cuh"
#include "q3_kernels.h"
#include "q3attn.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;   // 16 MiB per device
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

void* g_scratch_addr[kNoAllocMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (set up once per device).
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q3::record_cuda_error(e);
  if (dev < 0 || dev >= kNoAllocMaxDevices) return Q3_ERR_UNSUPPORTED;
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return q3::record_cuda_error(e);
    if (p == nullptr) return Q3_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return Q3_OK;
}

}  // namespace

extern "C" int q3_paged_decode_noalloc(const void* q, int64_t q_batch_stride, const void* k_new, const void* v_new,
                                       int64_t kv_new_batch_stride, void* k_pool, void* v_pool, int32_t num_pages,
                                       int32_t page_size, const int32_t* cache_seqlens, const int32_t* block_table,
                                       int64_t block_table_stride, int32_t max_pages_per_seat, int32_t batch,
                                       int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
                                       void* out, int64_t out_batch_stride, int32_t num_splits, void* stream) {
  // every check that needs no CUDA call first: a refused call queues nothing on the shared array
  int rc = q3::paged_decode_check_args(q, q_batch_stride, k_new, v_new, kv_new_batch_stride, k_pool, v_pool, num_pages,
                                       page_size, cache_seqlens, block_table, block_table_stride, max_pages_per_seat,
                                       batch, num_heads, num_kv_heads, head_dim, out, out_batch_stride, num_splits);
  if (rc != Q3_OK || batch == 0) return rc;
  const size_t need = q3_paged_decode_workspace_bytes(batch, num_splits);
  if (need == 0) return Q3_ERR_CUDA;
  if (need > kNoAllocScratchBytes) return Q3_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if ((rc = scratch_for_current_device(&scratch)) != Q3_OK) return rc;
  // the counters of seats 0..batch-1 must start at zero whatever an earlier (possibly failed) call left behind: they
  // are cleared on the stream after the remaining checks pass, right before the launch
  return q3::paged_decode_clearing_counters(q, q_batch_stride, k_new, v_new, kv_new_batch_stride, k_pool, v_pool,
                                            num_pages, page_size, cache_seqlens, block_table, block_table_stride,
                                            max_pages_per_seat, batch, num_heads, num_kv_heads, head_dim,
                                            softmax_scale, out, out_batch_stride, scratch, kNoAllocScratchBytes,
                                            num_splits, stream);
}
