// C ABI of q3attn (declared in include/q3attn.h): argument checks on the host, then one kernel launch per call.
#include <cstdio>
#include <cstring>

#include "q3_common.cuh"
#include "q3_kernels.h"
#include "q3attn.h"

namespace {

__device__ uint32_t g_status_word;   // OR of q3::kStatus* bits raised by any kernel of this library on this device

constexpr int kMaxDevices = 64;
thread_local char t_last_cuda_error[256] = "";
int g_decode_variant = 5;
int g_sm_count[kMaxDevices] = {0};
uint32_t* g_status_ptr[kMaxDevices] = {nullptr};

int record(cudaError_t e) {
  if (e == cudaSuccess) return Q3_OK;
  snprintf(t_last_cuda_error, sizeof(t_last_cuda_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return Q3_ERR_CUDA;
}

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return record(e);
  if (*dev < 0 || *dev >= kMaxDevices) return Q3_ERR_UNSUPPORTED;
  return Q3_OK;
}

int sm_count(int dev) {
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

// Device address of the status word of `dev` (cudaGetSymbolAddress with `dev` current).
int status_ptr(int dev, uint32_t** out) {
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_status_word);
    if (e != cudaSuccess) return record(e);
    g_status_ptr[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_status_ptr[dev];
  return Q3_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_family(int32_t nh, int32_t nkv, int32_t hd) {
  return (nh == q3::kQHeads && nkv == q3::kKvHeads && hd == q3::kHeadDim) ? Q3_OK : Q3_ERR_UNSUPPORTED;
}

long long decode_grid(int dev, int32_t batch, int32_t num_splits, int32_t max_pages, int32_t page_size, int variant) {
  const int rows = q3::decode_rows_per_chunk(variant);
  long long G = num_splits > 0 ? num_splits : static_cast<long long>(sm_count(dev)) * q3::decode_ctas_per_sm(variant);
  const long long max_chunks = static_cast<long long>(batch) * ((static_cast<long long>(max_pages) * page_size + rows - 1) / rows);
  if (max_pages > 0 && page_size > 0 && G > max_chunks) G = max_chunks;
  return G < 1 ? 1 : G;
}

// Decode workspace layout. The ticket counters (8 per seat) live in a front region whose size depends only on the
// workspace's byte count, never on the batch or the grid of a call, so partials written by one launch can never land
// where a later launch (any batch, any split count) keeps its counters. The counters are zero between launches.
constexpr size_t kSeatTicketBytes = q3::kKvHeads * sizeof(uint32_t);                                // 32
constexpr size_t kSlotMlBytes = q3::kKvHeads * q3::kGroup * 2 * sizeof(float);                      // 128
constexpr size_t kSlotOBytes = q3::kKvHeads * q3::kGroup * q3::kHeadDim * sizeof(float);            // 8192

size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct WsLayout {
  size_t counters, ml, o, end;
  bool fits;
};

WsLayout ws_layout(size_t bytes, int32_t batch, long long G) {
  WsLayout w;
  const size_t slots = static_cast<size_t>(G) + static_cast<size_t>(batch);
  w.counters = 0;
  w.ml = up256(kSeatTicketBytes * (bytes / (kSlotMlBytes + kSlotOBytes + kSeatTicketBytes)));
  w.o = w.ml + up256(slots * kSlotMlBytes);
  w.end = w.o + slots * kSlotOBytes;
  w.fits = kSeatTicketBytes * static_cast<size_t>(batch) <= w.ml && w.end <= bytes;
  return w;
}

size_t ws_bytes_needed(int32_t batch, long long G) {
  const size_t slots = static_cast<size_t>(G) + static_cast<size_t>(batch);
  size_t bytes = up256(slots * kSlotMlBytes) + slots * kSlotOBytes + kSeatTicketBytes * slots + 1024;
  while (!ws_layout(bytes, batch, G).fits) bytes += 4096;
  return bytes;
}

}  // namespace

extern "C" {

int q3_version(void) { return 100; }

const char* q3_error_string(int code) {
  switch (code) {
    case Q3_OK: return "ok";
    case Q3_ERR_INVALID: return "invalid argument";
    case Q3_ERR_UNSUPPORTED: return "unsupported shape (compiled for 16 q heads, 8 kv heads, head_dim 128)";
    case Q3_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case Q3_ERR_WORKSPACE: return "workspace missing or too small";
    case Q3_ERR_CUDA: return "CUDA runtime error";
    case Q3_ERR_SCRATCH_LIMIT: return "batch or split count beyond the fixed scratch of q3_paged_decode_noalloc";
    default: return "unknown error";
  }
}

const char* q3_last_cuda_error(void) { return t_last_cuda_error; }

int q3_device_sm_count(void) {
  int dev = 0;
  if (current_device(&dev) != Q3_OK) return 0;
  return sm_count(dev);
}

int q3_selftest_bounded_wait(uint64_t limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 100000000ull) return Q3_ERR_INVALID;
  int dev = 0, rc = current_device(&dev);
  if (rc != Q3_OK) return rc;
  uint32_t* p = nullptr;
  if ((rc = status_ptr(dev, &p)) != Q3_OK) return rc;
  return record(q3::launch_bounded_wait_selftest(p, limit_ns, static_cast<cudaStream_t>(stream)));
}

int q3_read_status(uint32_t* status_out, int clear) {
  int dev = 0, rc = current_device(&dev);
  if (rc != Q3_OK) return rc;
  uint32_t* p = nullptr;
  if ((rc = status_ptr(dev, &p)) != Q3_OK) return rc;
  uint32_t v = 0;
  cudaError_t e = cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return record(e);
  if (status_out) *status_out = v;
  if (clear) {
    e = cudaMemset(p, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return record(e);
  }
  return Q3_OK;
}

int q3_set_decode_variant(int variant) {
  const int prev = g_decode_variant;
  if (variant >= 0 && variant <= 5) g_decode_variant = variant;
  return prev;
}

int q3_paged_decode_resident_ctas(int variant) { return q3::decode_occupancy(variant); }

size_t q3_paged_decode_workspace_bytes(int32_t batch, int32_t num_splits) {
  int dev = 0;
  if (batch < 0 || current_device(&dev) != Q3_OK) return 0;
  // Upper bound over all block-table shapes and kernel configurations (the selected variant, and the default one that
  // q3_paged_decode_qkv falls back to): the grid is at most SMs x CTAs/SM (or num_splits) split slots.
  long long G = decode_grid(dev, batch, num_splits, 0, 0, g_decode_variant);
  const long long G0 = decode_grid(dev, batch, num_splits, 0, 0, 0);
  if (G0 > G) G = G0;
  return ws_bytes_needed(batch, G);
}

namespace {

bool norm_rope_ok(const q3_qk_norm_rope* nr) {
  return nr->q_norm_weight && nr->k_norm_weight && nr->cos && nr->sin && nr->rope_row_stride >= 0 &&
         nr->eps >= 0.f;
}

bool norm_rope_aligned(const q3_qk_norm_rope* nr) {
  return aligned(nr->q_norm_weight, 8) && aligned(nr->k_norm_weight, 8) && aligned(nr->cos, 8) &&
         aligned(nr->sin, 8) && (nr->rope_row_stride % 4) == 0;
}

// Argument checks of the decode entries that need no CUDA call (shapes, null pointers, strides, alignment).
int decode_check_args(const void* q, int64_t q_batch_stride, const void* k_new, const void* v_new,
                      int64_t kv_new_batch_stride, const q3_qk_norm_rope* nr, const void* k_pool, const void* v_pool,
                      int32_t num_pages, int32_t page_size, const int32_t* cache_seqlens, const int32_t* block_table,
                      int64_t block_table_stride, int32_t max_pages_per_seat, int32_t batch, int32_t num_heads,
                      int32_t num_kv_heads, int32_t head_dim, const void* out, int64_t out_batch_stride,
                      int32_t num_splits) {
  int rc = check_family(num_heads, num_kv_heads, head_dim);
  if (rc != Q3_OK) return rc;
  if (batch < 0 || num_pages <= 0 || page_size <= 0 || max_pages_per_seat <= 0 || num_splits < 0) return Q3_ERR_INVALID;
  if (batch == 0) return Q3_OK;
  if (!q || !k_pool || !v_pool || !cache_seqlens || !block_table || !out) return Q3_ERR_INVALID;
  if ((k_new == nullptr) != (v_new == nullptr)) return Q3_ERR_INVALID;
  if (nr && (!k_new || !norm_rope_ok(nr))) return Q3_ERR_INVALID;
  if (block_table_stride < max_pages_per_seat || q_batch_stride < q3::kQHeads * q3::kHeadDim ||
      out_batch_stride < q3::kQHeads * q3::kHeadDim)
    return Q3_ERR_INVALID;
  if (static_cast<long long>(max_pages_per_seat) * page_size > (1ll << 30)) return Q3_ERR_INVALID;
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(q, 16) || !aligned(out, 8) || (q_batch_stride % 8) ||
      (out_batch_stride % 4))
    return Q3_ERR_ALIGNMENT;
  if (k_new && (!aligned(k_new, 16) || !aligned(v_new, 16) || (kv_new_batch_stride % 8) ||
                kv_new_batch_stride < q3::kKvHeads * q3::kHeadDim))
    return Q3_ERR_ALIGNMENT;
  if (nr && !norm_rope_aligned(nr)) return Q3_ERR_ALIGNMENT;
  return Q3_OK;
}

// q3_paged_decode and q3_paged_decode_qkv: validation, workspace carving and launch. With nr set, q and k_new are raw
// projections and the kernel applies RMSNorm + RoPE (default configuration only). With clear_counters set, the ticket
// counters of the call's seats are zeroed on the stream right before the launch, after every check has passed (the
// workspace of the allocation-free entry may hold whatever an earlier call left).
int decode_common(const void* q, int64_t q_batch_stride, const void* k_new, const void* v_new,
                  int64_t kv_new_batch_stride, const q3_qk_norm_rope* nr, void* k_pool, void* v_pool,
                  int32_t num_pages, int32_t page_size, const int32_t* cache_seqlens, const int32_t* block_table,
                  int64_t block_table_stride, int32_t max_pages_per_seat, int32_t batch, int32_t num_heads,
                  int32_t num_kv_heads, int32_t head_dim, float softmax_scale, void* out, int64_t out_batch_stride,
                  void* workspace, size_t workspace_bytes, int32_t num_splits, void* stream,
                  bool clear_counters = false) {
  int rc = decode_check_args(q, q_batch_stride, k_new, v_new, kv_new_batch_stride, nr, k_pool, v_pool, num_pages,
                             page_size, cache_seqlens, block_table, block_table_stride, max_pages_per_seat, batch,
                             num_heads, num_kv_heads, head_dim, out, out_batch_stride, num_splits);
  if (rc != Q3_OK || batch == 0) return rc;
  int dev = 0;
  if ((rc = current_device(&dev)) != Q3_OK) return rc;
  // the fused q/k norm + RoPE form exists for variants 0 and 5
  const int variant = (nr && g_decode_variant != 5) ? 0 : g_decode_variant;
  const long long G = decode_grid(dev, batch, num_splits, max_pages_per_seat, page_size, variant);
  if (G > (1ll << 30)) return Q3_ERR_INVALID;
  const WsLayout w = ws_layout(workspace_bytes, batch, G);
  if (!workspace || !w.fits || !aligned(workspace, 256)) return Q3_ERR_WORKSPACE;
  uint32_t* st = nullptr;
  if ((rc = status_ptr(dev, &st)) != Q3_OK) return rc;

  q3::DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_batch_stride;
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  a.kv_new_stride = kv_new_batch_stride;
  a.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  a.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  a.seqlens = cache_seqlens;
  a.block_table = block_table;
  a.bt_stride = block_table_stride;
  a.max_pages = max_pages_per_seat;
  a.num_pages = num_pages;
  a.page_size = page_size;
  a.B = batch;
  a.scale_log2 = softmax_scale * q3::kLog2e;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_stride = out_batch_stride;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.counters = reinterpret_cast<uint32_t*>(ws + w.counters);
  a.ws_ml = reinterpret_cast<float*>(ws + w.ml);
  a.ws_o = reinterpret_cast<float*>(ws + w.o);
  a.status = st;
  // the full two-CTAs-per-SM grid gets the pair-weighted split (the kernel falls back to the uniform one when there
  // are too few chunks)
  a.pair_split = (num_splits <= 0 && q3::decode_ctas_per_sm(variant) == 2 && G == 2ll * sm_count(dev)) ? sm_count(dev) : 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (clear_counters) {
    cudaError_t e = cudaMemsetAsync(a.counters, 0, static_cast<size_t>(batch) * kSeatTicketBytes, s);
    if (e != cudaSuccess) return record(e);
  }
  if (nr) {
    a.qn_w = static_cast<const __nv_bfloat16*>(nr->q_norm_weight);
    a.kn_w = static_cast<const __nv_bfloat16*>(nr->k_norm_weight);
    a.rope_cos = static_cast<const __nv_bfloat16*>(nr->cos);
    a.rope_sin = static_cast<const __nv_bfloat16*>(nr->sin);
    a.rope_stride = nr->rope_row_stride;
    a.eps = nr->eps;
    return record(q3::launch_paged_decode_fused(a, static_cast<int>(G), variant, s));
  }
  return record(q3::launch_paged_decode(a, static_cast<int>(G), variant, s));
}

}  // namespace

}  // extern "C"

namespace q3 {

int record_cuda_error(cudaError_t e) { return record(e); }

int paged_decode_check_args(const void* q, int64_t q_batch_stride, const void* k_new, const void* v_new,
                            int64_t kv_new_batch_stride, const void* k_pool, const void* v_pool, int32_t num_pages,
                            int32_t page_size, const int32_t* cache_seqlens, const int32_t* block_table,
                            int64_t block_table_stride, int32_t max_pages_per_seat, int32_t batch, int32_t num_heads,
                            int32_t num_kv_heads, int32_t head_dim, const void* out, int64_t out_batch_stride,
                            int32_t num_splits) {
  return decode_check_args(q, q_batch_stride, k_new, v_new, kv_new_batch_stride, nullptr, k_pool, v_pool, num_pages,
                           page_size, cache_seqlens, block_table, block_table_stride, max_pages_per_seat, batch,
                           num_heads, num_kv_heads, head_dim, out, out_batch_stride, num_splits);
}

int paged_decode_clearing_counters(const void* q, int64_t q_batch_stride, const void* k_new, const void* v_new,
                                   int64_t kv_new_batch_stride, void* k_pool, void* v_pool, int32_t num_pages,
                                   int32_t page_size, const int32_t* cache_seqlens, const int32_t* block_table,
                                   int64_t block_table_stride, int32_t max_pages_per_seat, int32_t batch,
                                   int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
                                   void* out, int64_t out_batch_stride, void* workspace, size_t workspace_bytes,
                                   int32_t num_splits, void* stream) {
  return decode_common(q, q_batch_stride, k_new, v_new, kv_new_batch_stride, nullptr, k_pool, v_pool, num_pages,
                       page_size, cache_seqlens, block_table, block_table_stride, max_pages_per_seat, batch, num_heads,
                       num_kv_heads, head_dim, softmax_scale, out, out_batch_stride, workspace, workspace_bytes,
                       num_splits, stream, /*clear_counters=*/true);
}

}  // namespace q3

extern "C" {

int q3_paged_decode(const void* q, int64_t q_batch_stride, const void* k_new, const void* v_new,
                    int64_t kv_new_batch_stride, void* k_pool, void* v_pool, int32_t num_pages, int32_t page_size,
                    const int32_t* cache_seqlens, const int32_t* block_table, int64_t block_table_stride,
                    int32_t max_pages_per_seat, int32_t batch, int32_t num_heads, int32_t num_kv_heads,
                    int32_t head_dim, float softmax_scale, void* out, int64_t out_batch_stride, void* workspace,
                    size_t workspace_bytes, int32_t num_splits, void* stream) {
  return decode_common(q, q_batch_stride, k_new, v_new, kv_new_batch_stride, nullptr, k_pool, v_pool, num_pages,
                       page_size, cache_seqlens, block_table, block_table_stride, max_pages_per_seat, batch, num_heads,
                       num_kv_heads, head_dim, softmax_scale, out, out_batch_stride, workspace, workspace_bytes,
                       num_splits, stream);
}

int q3_paged_decode_qkv(const void* qkv, int64_t qkv_row_stride, const q3_qk_norm_rope* norm_rope, void* k_pool,
                        void* v_pool, int32_t num_pages, int32_t page_size, const int32_t* cache_seqlens,
                        const int32_t* block_table, int64_t block_table_stride, int32_t max_pages_per_seat,
                        int32_t batch, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
                        void* out, int64_t out_batch_stride, void* workspace, size_t workspace_bytes,
                        int32_t num_splits, void* stream) {
  if (!norm_rope) return Q3_ERR_INVALID;
  int rc = check_family(num_heads, num_kv_heads, head_dim);
  if (rc != Q3_OK) return rc;
  if (qkv_row_stride < (q3::kQHeads + 2 * q3::kKvHeads) * q3::kHeadDim) return Q3_ERR_INVALID;
  const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(qkv);
  const __nv_bfloat16* k_new = base ? base + q3::kQHeads * q3::kHeadDim : nullptr;
  const __nv_bfloat16* v_new = base ? base + (q3::kQHeads + q3::kKvHeads) * q3::kHeadDim : nullptr;
  return decode_common(qkv, qkv_row_stride, k_new, v_new, qkv_row_stride, norm_rope, k_pool, v_pool, num_pages,
                       page_size, cache_seqlens, block_table, block_table_stride, max_pages_per_seat, batch, num_heads,
                       num_kv_heads, head_dim, softmax_scale, out, out_batch_stride, workspace, workspace_bytes,
                       num_splits, stream);
}

static int append_common(q3::AppendArgs& a, const void* k, const void* v, int64_t row_stride, void* k_pool,
                         void* v_pool, int32_t nkv, int32_t hd, int32_t n_rows, void* stream) {
  if (n_rows < 0 || nkv <= 0 || hd <= 0) return Q3_ERR_INVALID;
  if (n_rows == 0) return Q3_OK;
  if (!k || !v || !k_pool || !v_pool) return Q3_ERR_INVALID;
  const int row_elems = nkv * hd;
  if (row_elems % 8 || row_stride < row_elems) return Q3_ERR_INVALID;
  if (!aligned(k, 16) || !aligned(v, 16) || !aligned(k_pool, 16) || !aligned(v_pool, 16) || (row_stride % 8))
    return Q3_ERR_ALIGNMENT;
  int dev = 0, rc = current_device(&dev);
  if (rc != Q3_OK) return rc;
  uint32_t* st = nullptr;
  if ((rc = status_ptr(dev, &st)) != Q3_OK) return rc;
  a.k_rows = static_cast<const __nv_bfloat16*>(k);
  a.v_rows = static_cast<const __nv_bfloat16*>(v);
  a.rows_stride = row_stride;
  a.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  a.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  a.row_elems = row_elems;
  a.n_rows = n_rows;
  a.status = st;
  return record(q3::launch_kv_append(a, sm_count(dev), static_cast<cudaStream_t>(stream)));
}

int q3_kv_append_slots(const void* k, const void* v, int64_t row_stride, void* k_pool, void* v_pool, int64_t pool_rows,
                       int32_t num_kv_heads, int32_t head_dim, const int64_t* slots, int32_t n_rows, void* stream) {
  if (n_rows > 0 && (!slots || pool_rows <= 0)) return Q3_ERR_INVALID;
  q3::AppendArgs a{};
  a.slots = slots;
  a.pool_rows = pool_rows;
  a.page_size = 1;
  return append_common(a, k, v, row_stride, k_pool, v_pool, num_kv_heads, head_dim, n_rows, stream);
}

int q3_kv_append_paged(const void* k, const void* v, int64_t row_stride, void* k_pool, void* v_pool, int32_t num_pages,
                       int32_t page_size, int32_t num_kv_heads, int32_t head_dim, const int32_t* positions,
                       const int32_t* seat_of_row, const int32_t* block_table, int64_t block_table_stride,
                       int32_t max_pages_per_seat, int32_t n_rows, void* stream) {
  if (n_rows > 0 && (!positions || !block_table || num_pages <= 0 || page_size <= 0 || max_pages_per_seat <= 0 ||
                     block_table_stride < max_pages_per_seat))
    return Q3_ERR_INVALID;
  q3::AppendArgs a{};
  a.positions = positions;
  a.seat_of_row = seat_of_row;
  a.block_table = block_table;
  a.bt_stride = block_table_stride;
  a.max_pages = max_pages_per_seat;
  a.page_size = page_size;
  a.pool_rows = static_cast<long long>(num_pages) * page_size;
  return append_common(a, k, v, row_stride, k_pool, v_pool, num_kv_heads, head_dim, n_rows, stream);
}

static int cp_common(q3::CpArgs& a, const void* q, int64_t q_batch_stride, void* K, void* V, int64_t kb, int64_t kh,
                     int64_t ks, int64_t vb, int64_t vh, int64_t vs, int32_t batch, int32_t n_slots, int32_t n_live,
                     float scale, void* out, int64_t out_stride, void* stream) {
  if (batch < 0 || n_slots <= 0 || n_live < 1 || n_live > n_slots) return Q3_ERR_INVALID;
  if (n_live > 16) return Q3_ERR_UNSUPPORTED;
  if (batch == 0) return Q3_OK;
  if (!q || !K || !V || !out) return Q3_ERR_INVALID;
  if (q_batch_stride < q3::kQHeads * q3::kHeadDim || out_stride < q3::kQHeads * q3::kHeadDim) return Q3_ERR_INVALID;
  int dev = 0, rc;
  if ((rc = current_device(&dev)) != Q3_OK) return rc;
  uint32_t* st = nullptr;
  if ((rc = status_ptr(dev, &st)) != Q3_OK) return rc;
  a.status = st;
  if (!aligned(q, 8) || !aligned(K, 8) || !aligned(V, 8) || !aligned(out, 8) || (q_batch_stride % 4) || (out_stride % 4) ||
      (kb % 4) || (kh % 4) || (ks % 4) || (vb % 4) || (vh % 4) || (vs % 4))
    return Q3_ERR_ALIGNMENT;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_batch_stride;
  a.K = static_cast<__nv_bfloat16*>(K);
  a.V = static_cast<__nv_bfloat16*>(V);
  a.sk_b = kb; a.sk_h = kh; a.sk_s = ks;
  a.sv_b = vb; a.sv_h = vh; a.sv_s = vs;
  a.B = batch;
  a.n_live = n_live;
  // one bulk copy per (seat, head) when its live slots are one contiguous 16-byte aligned range
  a.bulk = (ks == q3::kHeadDim && vs == q3::kHeadDim && aligned(K, 16) && aligned(V, 16) && (kb % 8) == 0 &&
            (kh % 8) == 0 && (vb % 8) == 0 && (vh % 8) == 0) ? 1 : 0;
  a.scale_log2 = scale * q3::kLog2e;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_stride = out_stride;
  return record(q3::launch_cp_attn(a, static_cast<cudaStream_t>(stream)));
}

int q3_cp_attn(const void* q, int64_t q_batch_stride, const void* K, const void* V, int64_t k_batch_stride,
               int64_t k_head_stride, int64_t k_slot_stride, int64_t v_batch_stride, int64_t v_head_stride,
               int64_t v_slot_stride, int32_t batch, int32_t n_slots, int32_t n_live, float softmax_scale, void* out,
               int64_t out_batch_stride, void* stream) {
  q3::CpArgs a{};
  return cp_common(a, q, q_batch_stride, const_cast<void*>(K), const_cast<void*>(V), k_batch_stride, k_head_stride,
                   k_slot_stride, v_batch_stride, v_head_stride, v_slot_stride, batch, n_slots, n_live, softmax_scale,
                   out, out_batch_stride, stream);
}

int q3_cp_step(const void* q, int64_t q_batch_stride, const void* k_new, const void* v_new, int64_t kv_new_batch_stride,
               void* K, void* V, int64_t k_batch_stride, int64_t k_head_stride, int64_t k_slot_stride,
               int64_t v_batch_stride, int64_t v_head_stride, int64_t v_slot_stride, int32_t batch, int32_t n_slots,
               int32_t slot, float softmax_scale, void* out, int64_t out_batch_stride, void* stream) {
  if (batch > 0 && (!k_new || !v_new || kv_new_batch_stride < q3::kKvHeads * q3::kHeadDim)) return Q3_ERR_INVALID;
  if (batch > 0 && (!aligned(k_new, 8) || !aligned(v_new, 8) || (kv_new_batch_stride % 4))) return Q3_ERR_ALIGNMENT;
  q3::CpArgs a{};
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  a.kv_new_stride = kv_new_batch_stride;
  return cp_common(a, q, q_batch_stride, K, V, k_batch_stride, k_head_stride, k_slot_stride, v_batch_stride,
                   v_head_stride, v_slot_stride, batch, n_slots, slot + 1, softmax_scale, out, out_batch_stride, stream);
}

int q3_cp_step_qkv(const void* qkv, int64_t qkv_row_stride, const q3_qk_norm_rope* norm_rope, void* K, void* V,
                   int64_t k_batch_stride, int64_t k_head_stride, int64_t k_slot_stride, int64_t v_batch_stride,
                   int64_t v_head_stride, int64_t v_slot_stride, int32_t batch, int32_t n_slots, int32_t slot,
                   float softmax_scale, void* out, int64_t out_batch_stride, void* stream) {
  if (!norm_rope || !norm_rope_ok(norm_rope)) return Q3_ERR_INVALID;
  if (qkv_row_stride < (q3::kQHeads + 2 * q3::kKvHeads) * q3::kHeadDim) return Q3_ERR_INVALID;
  if (!norm_rope_aligned(norm_rope)) return Q3_ERR_ALIGNMENT;
  const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(qkv);
  q3::CpArgs a{};
  a.k_new = base ? base + q3::kQHeads * q3::kHeadDim : nullptr;
  a.v_new = base ? base + (q3::kQHeads + q3::kKvHeads) * q3::kHeadDim : nullptr;
  a.kv_new_stride = qkv_row_stride;
  a.qn_w = static_cast<const __nv_bfloat16*>(norm_rope->q_norm_weight);
  a.kn_w = static_cast<const __nv_bfloat16*>(norm_rope->k_norm_weight);
  a.rope_cos = static_cast<const __nv_bfloat16*>(norm_rope->cos);
  a.rope_sin = static_cast<const __nv_bfloat16*>(norm_rope->sin);
  a.rope_stride = norm_rope->rope_row_stride;
  a.eps = norm_rope->eps;
  return cp_common(a, qkv, qkv_row_stride, K, V, k_batch_stride, k_head_stride, k_slot_stride, v_batch_stride,
                   v_head_stride, v_slot_stride, batch, n_slots, slot + 1, softmax_scale, out, out_batch_stride, stream);
}

int q3_sample_topk(const q3_sampler* p, void* stream) {
  if (!p) return Q3_ERR_INVALID;
  if (p->batch < 0) return Q3_ERR_INVALID;
  if (p->batch == 0) return Q3_OK;
  if (p->vocab < 1 || p->vocab > 4096 || p->top_k < 1 || p->top_k > q3::kSampleMaxTopK || p->top_k > p->vocab)
    return p->vocab > 4096 || p->top_k > q3::kSampleMaxTopK ? Q3_ERR_UNSUPPORTED : Q3_ERR_INVALID;
  if (p->top_k > 1 && !(p->temperature > 0.f)) return Q3_ERR_INVALID;
  if (!p->logits || !p->rng_state || !p->out_ids || (p->logits_dtype != 0 && p->logits_dtype != 1)) return Q3_ERR_INVALID;
  if (p->row_stride < p->vocab || p->out_stride < 1) return Q3_ERR_INVALID;
  if ((p->seen || p->ngen) && !p->seat) return Q3_ERR_INVALID;
  if (p->seen && p->seen_row_stride < p->vocab) return Q3_ERR_INVALID;
  if (p->emb && (!p->emb_out || p->emb_dim <= 0 || p->emb_row_stride < p->emb_dim || p->emb_out_row_stride < p->emb_dim))
    return Q3_ERR_INVALID;
  if (!aligned(p->rng_state, 8) || (p->emb && (!aligned(p->emb, 8) || !aligned(p->emb_out, 8) || (p->emb_dim % 4) ||
                                              (p->emb_row_stride % 4) || (p->emb_out_row_stride % 4))))
    return Q3_ERR_ALIGNMENT;
  if (p->batch > 2147483647) return Q3_ERR_INVALID;
  q3::SampleArgs a{};
  a.logits = p->logits;
  a.logits_bf16 = p->logits_dtype == 0;
  a.row_stride = p->row_stride;
  a.B = p->batch;
  a.V = p->vocab;
  a.k = p->top_k;
  a.inv_temp = p->top_k > 1 ? 1.f / p->temperature : 1.f;
  a.seen = p->seen;
  a.seen_stride = p->seen_row_stride;
  a.seat = p->seat;
  a.rep = p->repetition_penalty;
  a.bias = p->bias;
  a.ngen = p->ngen;
  a.min_new = p->min_new;
  a.eos = p->eos_id;
  a.seed = p->seed;
  a.rng_state = reinterpret_cast<unsigned long long*>(p->rng_state);
  a.out_ids = p->out_ids;
  a.out_stride = p->out_stride;
  a.emb = static_cast<const __nv_bfloat16*>(p->emb);
  a.emb_stride = p->emb_row_stride;
  a.emb_dim = p->emb_dim;
  a.emb_out = static_cast<__nv_bfloat16*>(p->emb_out);
  a.emb_out_stride = p->emb_out_row_stride;
  return record(q3::launch_sample_topk(a, static_cast<cudaStream_t>(stream)));
}

int q3_kv_copy_prefix(const void* k_src, const void* v_src, int64_t src_layer_stride, int64_t src_slot_stride,
                      const uint64_t* k_pools, const uint64_t* v_pools, int32_t num_layers, int64_t pool_rows,
                      int32_t page_size, int32_t num_kv_heads, int32_t head_dim, const int64_t* seat,
                      const int64_t* slot, int32_t batch, int32_t prefix_len, const int32_t* block_table,
                      int64_t block_table_stride, int32_t max_pages_per_seat, void* stream) {
  if (num_layers < 0 || batch < 0 || prefix_len < 0 || num_kv_heads <= 0 || head_dim <= 0) return Q3_ERR_INVALID;
  if (num_layers == 0 || batch == 0 || prefix_len == 0) return Q3_OK;
  const int row_elems = num_kv_heads * head_dim;
  if (!k_src || !v_src || !k_pools || !v_pools || !seat || !slot || !block_table || pool_rows <= 0 || page_size <= 0 ||
      max_pages_per_seat <= 0 || block_table_stride < max_pages_per_seat || row_elems % 8)
    return Q3_ERR_INVALID;
  if (src_layer_stride < 0 || src_slot_stride < 0) return Q3_ERR_INVALID;
  if (!aligned(k_src, 16) || !aligned(v_src, 16) || (src_layer_stride % 8) || (src_slot_stride % 8) ||
      !aligned(k_pools, 8) || !aligned(v_pools, 8))
    return Q3_ERR_ALIGNMENT;
  int dev = 0, rc = current_device(&dev);
  if (rc != Q3_OK) return rc;
  uint32_t* st = nullptr;
  if ((rc = status_ptr(dev, &st)) != Q3_OK) return rc;
  q3::PrefixCopyArgs a{};
  a.k_src = static_cast<const __nv_bfloat16*>(k_src);
  a.v_src = static_cast<const __nv_bfloat16*>(v_src);
  a.src_layer_stride = src_layer_stride;
  a.src_slot_stride = src_slot_stride;
  a.k_pools = reinterpret_cast<const unsigned long long*>(k_pools);
  a.v_pools = reinterpret_cast<const unsigned long long*>(v_pools);
  a.L = num_layers;
  a.pool_rows = pool_rows;
  a.page_size = page_size;
  a.row_elems = row_elems;
  a.seat = seat;
  a.slot = slot;
  a.B = batch;
  a.prefix_len = prefix_len;
  a.block_table = block_table;
  a.bt_stride = block_table_stride;
  a.max_pages = max_pages_per_seat;
  a.status = st;
  return record(q3::launch_kv_copy_prefix(a, sm_count(dev), static_cast<cudaStream_t>(stream)));
}

int q3_add_rms_norm(void* x, int64_t x_row_stride, const void* residual, int64_t residual_row_stride,
                    const void* weight, void* out, int64_t out_row_stride, int64_t rows, int32_t hidden, float eps,
                    void* stream) {
  if (rows < 0) return Q3_ERR_INVALID;
  if (hidden != 1024 && hidden != 2048) return Q3_ERR_UNSUPPORTED;
  if (rows == 0) return Q3_OK;
  if (!x || !weight || !out || x_row_stride < hidden || out_row_stride < hidden || !(eps >= 0.f) ||
      (residual && residual_row_stride < hidden) || rows > (1ll << 31) * 4)
    return Q3_ERR_INVALID;
  if (!aligned(x, 16) || !aligned(weight, 16) || !aligned(out, 16) || (x_row_stride % 8) || (out_row_stride % 8) ||
      (residual && (!aligned(residual, 16) || (residual_row_stride % 8))))
    return Q3_ERR_ALIGNMENT;
  q3::RowNormArgs a{};
  a.x = static_cast<__nv_bfloat16*>(x);
  a.x_stride = x_row_stride;
  a.r = static_cast<const __nv_bfloat16*>(residual);
  a.r_stride = residual_row_stride;
  a.w = static_cast<const __nv_bfloat16*>(weight);
  a.y = static_cast<__nv_bfloat16*>(out);
  a.y_stride = out_row_stride;
  a.rows = rows;
  a.H = hidden;
  a.eps = eps;
  return record(q3::launch_add_rms_norm(a, static_cast<cudaStream_t>(stream)));
}

int q3_silu_mul(const void* gate_up, int64_t gate_up_row_stride, void* out, int64_t out_row_stride, int64_t rows,
                int32_t ffn, void* stream) {
  if (rows < 0 || ffn <= 0 || (ffn % 8)) return Q3_ERR_INVALID;
  if (rows == 0) return Q3_OK;
  if (!gate_up || !out || gate_up_row_stride < 2ll * ffn || out_row_stride < ffn) return Q3_ERR_INVALID;
  if (!aligned(gate_up, 16) || !aligned(out, 16) || (gate_up_row_stride % 8) || (out_row_stride % 8))
    return Q3_ERR_ALIGNMENT;
  int dev = 0, rc = current_device(&dev);
  if (rc != Q3_OK) return rc;
  q3::SiluMulArgs a{};
  a.gu = static_cast<const __nv_bfloat16*>(gate_up);
  a.gu_stride = gate_up_row_stride;
  a.y = static_cast<__nv_bfloat16*>(out);
  a.y_stride = out_row_stride;
  a.rows = rows;
  a.F = ffn;
  return record(q3::launch_silu_mul(a, sm_count(dev), static_cast<cudaStream_t>(stream)));
}

int q3_qk_norm_rope_rows(void* qkv, int64_t qkv_row_stride, const q3_qk_norm_rope* norm_rope, int64_t rows,
                         void* stream) {
  if (rows < 0 || !norm_rope || !norm_rope_ok(norm_rope)) return Q3_ERR_INVALID;
  if (rows == 0) return Q3_OK;
  if (!qkv || qkv_row_stride < (q3::kQHeads + 2 * q3::kKvHeads) * q3::kHeadDim) return Q3_ERR_INVALID;
  if (!aligned(qkv, 8) || (qkv_row_stride % 4) || !norm_rope_aligned(norm_rope)) return Q3_ERR_ALIGNMENT;
  q3::QkNormRopeArgs a{};
  a.qkv = static_cast<__nv_bfloat16*>(qkv);
  a.qkv_stride = qkv_row_stride;
  a.rows = rows;
  a.qn_w = static_cast<const __nv_bfloat16*>(norm_rope->q_norm_weight);
  a.kn_w = static_cast<const __nv_bfloat16*>(norm_rope->k_norm_weight);
  a.rope_cos = static_cast<const __nv_bfloat16*>(norm_rope->cos);
  a.rope_sin = static_cast<const __nv_bfloat16*>(norm_rope->sin);
  a.rope_stride = norm_rope->rope_row_stride;
  a.eps = norm_rope->eps;
  return record(q3::launch_qk_norm_rope(a, static_cast<cudaStream_t>(stream)));
}

int q3_set_ring_frame_kernel(int kernel) {
  const int prev = q3::g_ring_frame_kernel;
  if (kernel >= 0 && kernel <= 6) q3::g_ring_frame_kernel = kernel;
  return prev;
}

int q3_set_ring_chunk_kernel(int kernel) {
  const int prev = q3::g_ring_chunk_kernel;
  if (kernel >= 0 && kernel <= 4) q3::g_ring_chunk_kernel = kernel;
  return prev;
}

int q3_ring_window_attn(const void* q, const void* k_new, const void* v_new, int64_t qkv_batch_stride,
                        int64_t qkv_frame_stride, void* k_ring, void* v_ring, int64_t ring_stream_stride,
                        int64_t ring_slot_stride, const int64_t* ring_rows, const int64_t* pos, int32_t batch,
                        int32_t n, int32_t heads, int32_t head_dim, int32_t ring, int32_t past, float scale,
                        int32_t write_new, void* out, int64_t out_batch_stride, int64_t out_frame_stride,
                        void* stream) {
  if (batch < 0 || n < 0 || heads <= 0 || ring <= 0 || past < 0) return Q3_ERR_INVALID;
  if ((head_dim != 64 && head_dim != 128) || ring > q3::kRingMaxSlots || n > q3::kRingMaxChunk) return Q3_ERR_UNSUPPORTED;
  if (n > ring - past) return Q3_ERR_INVALID;               // the chunk's ring slots must lie outside every window
  if (batch == 0 || n == 0) return Q3_OK;
  if (!q || !k_new || !v_new || !k_ring || !v_ring || !ring_rows || !pos || !out || batch > 2147483647) return Q3_ERR_INVALID;
  if (qkv_frame_stride < static_cast<int64_t>(heads) * head_dim || ring_slot_stride < static_cast<int64_t>(heads) * head_dim ||
      out_frame_stride < static_cast<int64_t>(heads) * head_dim || qkv_batch_stride < 0 || ring_stream_stride < 0 ||
      out_batch_stride < 0)
    return Q3_ERR_INVALID;
  if (!aligned(q, 16) || !aligned(k_new, 16) || !aligned(v_new, 16) || !aligned(k_ring, 16) || !aligned(v_ring, 16) ||
      !aligned(out, 4) || (qkv_batch_stride % 8) || (qkv_frame_stride % 8) || (ring_stream_stride % 8) ||
      (ring_slot_stride % 8) || (out_batch_stride % 2) || (out_frame_stride % 2))
    return Q3_ERR_ALIGNMENT;
  q3::RingArgs a{};
  a.q = static_cast<const __half*>(q);
  a.k_new = static_cast<const __half*>(k_new);
  a.v_new = static_cast<const __half*>(v_new);
  a.qkv_batch_stride = qkv_batch_stride;
  a.qkv_frame_stride = qkv_frame_stride;
  a.k_ring = static_cast<__half*>(k_ring);
  a.v_ring = static_cast<__half*>(v_ring);
  a.ring_stream_stride = ring_stream_stride;
  a.ring_slot_stride = ring_slot_stride;
  a.ring_rows = ring_rows;
  a.pos = pos;
  a.B = batch;
  a.n = n;
  a.H = heads;
  a.hd = head_dim;
  a.ring = ring;
  a.past = past;
  a.scale = scale;
  a.write_new = write_new;
  a.out = static_cast<__half*>(out);
  a.out_batch_stride = out_batch_stride;
  a.out_frame_stride = out_frame_stride;
  int dev = 0, rc;
  if ((rc = current_device(&dev)) != Q3_OK) return rc;
  if ((rc = status_ptr(dev, &a.status)) != Q3_OK) return rc;
  return record(q3::launch_ring_attn(a, static_cast<cudaStream_t>(stream)));
}

int q3_set_prefill_kernel(int kernel) {
  const int prev = q3::g_prefill_kernel;
  if (kernel == 0 || kernel == 1) q3::g_prefill_kernel = kernel;
  return prev;
}

int q3_prefill(const void* q, int64_t q_row_stride, int64_t q_rows, const void* k, const void* v,
               int64_t kv_row_stride, int64_t kv_rows,
               const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t num_seqs, int32_t max_seqlen_q,
               const int32_t* prefix_lens, const int32_t* seat_ids, void* k_pool, void* v_pool, int32_t num_pages,
               int32_t page_size, const int32_t* block_table, int64_t block_table_stride, int32_t max_pages_per_seat,
               int32_t write_kv, int32_t causal, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
               float softmax_scale, void* out, int64_t out_row_stride, void* stream) {
  int rc = check_family(num_heads, num_kv_heads, head_dim);
  if (rc != Q3_OK) return rc;
  if (num_seqs < 0 || max_seqlen_q < 0 || q_rows < 0 || kv_rows < 0) return Q3_ERR_INVALID;
  if (num_seqs == 0 || q_rows == 0) return Q3_OK;
  if (!q || !k || !v || !cu_seqlens_q || !cu_seqlens_k || !out) return Q3_ERR_INVALID;
  if (q_row_stride < q3::kQHeads * q3::kHeadDim || out_row_stride < q3::kQHeads * q3::kHeadDim ||
      kv_row_stride < q3::kKvHeads * q3::kHeadDim)
    return Q3_ERR_INVALID;
  const bool paged = (prefix_lens != nullptr) || write_kv;
  if (paged && (!k_pool || !v_pool || !block_table || num_pages <= 0 || page_size <= 0 || max_pages_per_seat <= 0 ||
                block_table_stride < max_pages_per_seat))
    return Q3_ERR_INVALID;
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16) || (q_row_stride % 8) ||
      (kv_row_stride % 8) || (out_row_stride % 8) || (paged && (!aligned(k_pool, 16) || !aligned(v_pool, 16))))
    return Q3_ERR_ALIGNMENT;
  if (static_cast<long long>(max_seqlen_q + 63) / 64 > 65535 || num_seqs > 65535) return Q3_ERR_INVALID;
  int dev = 0;
  if ((rc = current_device(&dev)) != Q3_OK) return rc;
  uint32_t* st = nullptr;
  if ((rc = status_ptr(dev, &st)) != Q3_OK) return rc;
  q3::PrefillArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_row_stride;
  a.q_rows = q_rows;
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.kv_stride = kv_row_stride;
  a.kv_rows = kv_rows;
  a.cu_q = cu_seqlens_q;
  a.cu_k = cu_seqlens_k;
  a.num_seqs = num_seqs;
  a.max_seqlen_q = max_seqlen_q;
  a.prefix_lens = prefix_lens;
  a.seat_ids = seat_ids;
  a.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  a.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  a.num_pages = num_pages;
  a.page_size = page_size;
  a.block_table = block_table;
  a.bt_stride = block_table_stride;
  a.max_pages = max_pages_per_seat;
  a.write_kv = write_kv ? 1 : 0;
  a.causal = causal ? 1 : 0;
  a.scale_log2 = softmax_scale * q3::kLog2e;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_stride = out_row_stride;
  a.status = st;
  return record(q3::launch_prefill(a, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
