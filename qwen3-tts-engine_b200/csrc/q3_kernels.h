// Internal launch interface between the C-ABI layer (capi.cu) and the kernels. Not installed; include/q3attn.h is the
// public boundary.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace q3 {

struct DecodeArgs {
  const __nv_bfloat16* q;          // [B, 16, 128] rows, batch stride q_stride (elements)
  long long q_stride;
  const __nv_bfloat16* k_new;      // [B, 8, 128] or nullptr (no append)
  const __nv_bfloat16* v_new;
  long long kv_new_stride;
  __nv_bfloat16* k_pool;           // [num_pages, page_size, 8, 128] contiguous
  __nv_bfloat16* v_pool;
  const int32_t* seqlens;          // [B] tokens in the cache before the append (== tokens attended without append)
  const int32_t* block_table;      // [B, bt_stride] (first max_pages entries of a row are usable)
  long long bt_stride;
  int max_pages;
  int num_pages;
  int page_size;
  int B;
  float scale_log2;                // softmax_scale * log2(e)
  __nv_bfloat16* out;              // [B, 16, 128] rows, batch stride out_stride
  long long out_stride;
  float* ws_o;                     // [(G + B), 8, 2, 128] fp32 partial outputs
  float* ws_ml;                    // [(G + B), 8, 2, 2] fp32 (running max, running sum)
  uint32_t* counters;              // [B, 8] zero between launches
  uint32_t* status;
  int pair_split = 0;              // SM count when the grid is two CTAs per SM on every SM (pair-weighted split)
  int split_slots = 0;             // the dedicated-producer kernel: chunk streams of the split (two per CTA)
  // Fused q/k RMSNorm + RoPE (the kernel instantiated with FUSE): q rows and k_new rows are raw projections.
  const __nv_bfloat16* qn_w = nullptr;     // [128]
  const __nv_bfloat16* kn_w = nullptr;     // [128]
  const __nv_bfloat16* rope_cos = nullptr; // row b at b * rope_stride, [128] each
  const __nv_bfloat16* rope_sin = nullptr;
  long long rope_stride = 0;
  float eps = 1e-6f;
};

// One CTA whose bounded mbarrier wait expires after limit_ns and raises the wait-timeout bit in *status.
cudaError_t launch_bounded_wait_selftest(uint32_t* status, unsigned long long limit_ns, cudaStream_t stream);

int decode_rows_per_chunk(int variant);
int decode_ctas_per_sm(int variant);
int decode_occupancy(int variant);   // resident CTAs per SM measured by the runtime (-1 on error)
cudaError_t launch_paged_decode(const DecodeArgs& a, int grid, int variant, cudaStream_t stream);
// The q/k RMSNorm + RoPE fused in (a.qn_w etc. set, k_new required): variant 5 (dedicated producers) or, for any other
// variant, variant 0.
cudaError_t launch_paged_decode_fused(const DecodeArgs& a, int grid, int variant, cudaStream_t stream);

struct AppendArgs {
  const __nv_bfloat16* k_rows;     // [n_rows, row_elems] with row stride rows_stride (elements)
  const __nv_bfloat16* v_rows;
  long long rows_stride;
  __nv_bfloat16* k_pool;           // [num_pages * page_size, row_elems]
  __nv_bfloat16* v_pool;
  long long pool_rows;             // num_pages * page_size
  int page_size;
  int row_elems;                   // nkv * head_dim
  int n_rows;
  const int64_t* slots;            // flat destination row per input row, or nullptr
  const int32_t* positions;        // token position per input row (paged mode)
  const int32_t* seat_of_row;      // seat per input row (paged mode; nullptr = row i belongs to seat i)
  const int32_t* block_table;
  long long bt_stride;
  int max_pages;
  uint32_t* status;
};

cudaError_t launch_kv_append(const AppendArgs& a, int num_sms, cudaStream_t stream);

struct PrefixCopyArgs {
  const __nv_bfloat16* k_src;      // row (l, slot, r) at l * src_layer_stride + slot * src_slot_stride + r * row_elems
  const __nv_bfloat16* v_src;
  long long src_layer_stride, src_slot_stride;
  const unsigned long long* k_pools;   // [L] device addresses of each layer's [pool_rows, row_elems] pool
  const unsigned long long* v_pools;
  int L;
  long long pool_rows;
  int page_size, row_elems;
  const int64_t* seat;             // [B] destination seat
  const int64_t* slot;             // [B] prefix slot
  int B, prefix_len;
  const int32_t* block_table;
  long long bt_stride;
  int max_pages;
  uint32_t* status;
};

cudaError_t launch_kv_copy_prefix(const PrefixCopyArgs& a, int num_sms, cudaStream_t stream);

struct CpArgs {
  const __nv_bfloat16* q;          // [B, 16, 128] rows, batch stride q_stride
  long long q_stride;
  const __nv_bfloat16* k_new;      // [B, 8, 128] or nullptr (attention only)
  const __nv_bfloat16* v_new;
  long long kv_new_stride;
  __nv_bfloat16* K;                // [B, 8, S, 128] with strides (elements) sk_b, sk_h, sk_s; innermost contiguous
  __nv_bfloat16* V;
  long long sk_b, sk_h, sk_s;
  long long sv_b, sv_h, sv_s;
  int B;
  int n_live;                      // slots attended: 1..16; with k_new the new row lands in slot n_live - 1
  int bulk;                        // 1: slot rows contiguous (stride 128) and every (seat, head) base 16-byte aligned
  uint32_t* status;                // error bits (a bulk-copy wait that gave up)
  float scale_log2;
  __nv_bfloat16* out;              // [B, 16*128] rows, batch stride out_stride
  long long out_stride;
  // Fused q/k RMSNorm + RoPE (nullptr: q and k_new are used as given); k_new required when set.
  const __nv_bfloat16* qn_w = nullptr;
  const __nv_bfloat16* kn_w = nullptr;
  const __nv_bfloat16* rope_cos = nullptr;
  const __nv_bfloat16* rope_sin = nullptr;
  long long rope_stride = 0;
  float eps = 1e-6f;
};

cudaError_t launch_cp_attn(const CpArgs& a, cudaStream_t stream);

constexpr int kSampleMaxTopK = 64;
struct SampleArgs {
  const void* logits;              // [B, V] rows (bf16 or fp32), row stride row_stride (elements)
  int logits_bf16;
  long long row_stride;
  int B, V, k;                     // V <= 4096, 1 <= k <= min(64, V)
  float inv_temp;
  const uint8_t* seen;             // optional [S, V] bool rows (repetition penalty), row = seat[b]
  long long seen_stride;
  const int64_t* seat;             // [B] row of seen / ngen for batch row b (needed with seen or ngen)
  float rep;
  const float* bias;               // optional [V] additive (the suppress row)
  const int64_t* ngen;             // optional [S]: EOS is masked while ngen[seat[b]] < min_new
  int min_new, eos;
  unsigned long long seed;
  unsigned long long* rng_state;   // device [2]: launch index, finish ticket
  int64_t* out_ids;                // [B] at stride out_stride
  long long out_stride;
  const __nv_bfloat16* emb;        // optional [*, emb_dim] table: row out_ids[b] copied to emb_out row b
  long long emb_stride;
  int emb_dim;
  __nv_bfloat16* emb_out;
  long long emb_out_stride;
};

cudaError_t launch_sample_topk(const SampleArgs& a, cudaStream_t stream);

struct RowNormArgs {
  __nv_bfloat16* x;                // [rows, H] residual stream (updated in place when r is given)
  long long x_stride;
  const __nv_bfloat16* r;          // optional [rows, H] added to x first
  long long r_stride;
  const __nv_bfloat16* w;          // [H]
  __nv_bfloat16* y;                // [rows, H] normalised output
  long long y_stride;
  long long rows;
  int H;                           // 1024 or 2048
  float eps;
};
cudaError_t launch_add_rms_norm(const RowNormArgs& a, cudaStream_t stream);

struct SiluMulArgs {
  const __nv_bfloat16* gu;         // [rows, 2F]: gate | up
  long long gu_stride;
  __nv_bfloat16* y;                // [rows, F]
  long long y_stride;
  long long rows;
  int F;
};
cudaError_t launch_silu_mul(const SiluMulArgs& a, int num_sms, cudaStream_t stream);

struct QkNormRopeArgs {
  __nv_bfloat16* qkv;              // [rows, (16 + 8 + 8) * 128]: q and k heads rewritten in place
  long long qkv_stride;
  long long rows;
  const __nv_bfloat16* qn_w;
  const __nv_bfloat16* kn_w;
  const __nv_bfloat16* rope_cos;   // row r at r * rope_stride
  const __nv_bfloat16* rope_sin;
  long long rope_stride;
  float eps;
};
cudaError_t launch_qk_norm_rope(const QkNormRopeArgs& a, cudaStream_t stream);

constexpr int kRingMaxChunk = 17;     // frames per call: at most RING - PAST (88 - 71) in the reference
constexpr int kRingMaxSlots = 128;
struct RingArgs {
  const __half* q;                 // [B, n, H, hd] rotated queries (batch / frame strides; heads hd apart)
  const __half* k_new;             // [B, n, H, hd] the chunk's rotated keys
  const __half* v_new;
  long long qkv_batch_stride, qkv_frame_stride;
  __half* k_ring;                  // stream row r, slot s, head h at r * ring_stream_stride + s * ring_slot_stride + h*hd
  __half* v_ring;
  long long ring_stream_stride, ring_slot_stride;
  const int64_t* ring_rows;        // [B] ring row of each batch entry
  const int64_t* pos;              // [B] frames decoded before this chunk
  int B, n, H, hd, ring, past;
  float scale;
  int write_new;
  __half* out;                     // [B, n, H * hd]
  long long out_batch_stride, out_frame_stride;
  uint32_t* status;                // error bits (a staging wait that gave up)
  // set by launch_ring_attn: the multiply-high reciprocal of ring (ceil(2^(63 + l) / ring), l = ceil(log2 ring)) and
  // l - 1, through which the streaming kernel takes positions modulo the ring
  unsigned long long ring_magic;
  int ring_shift;
};
size_t ring_smem_bytes(int ring, int past, int hd, int n);
cudaError_t launch_ring_attn(const RingArgs& a, cudaStream_t stream);
// Which one-frame ring kernel launch_ring_attn uses: 6 = nothing staged, 4 / 8 warps per (stream, head) of 64 / 128
// dims loading straight into registers (default; windows past 79 rows go to 2); 2 = scalar math, one warp per head, 4 x 64 / 2 x 128
// heads per CTA; 1 = scalar math, one CTA per (stream, head) (also every call another selection does not fit);
// 0 / 3 / 4 = tensor cores, one warp per head, 4 / 2 / 1 heads of 64 per CTA; 5 = the persistent TMA pipeline.
extern int g_ring_frame_kernel;
// Which kernel runs chunks of 2 .. 17 frames: 1 = one CTA per (stream, head) (default, also every call another
// selection does not fit); 0 / 2 / 3 = tensor cores, one warp per head, 2 / 4 / 1 heads of 64 per CTA; 4 = the
// persistent TMA pipeline (2 .. 8 frames).
extern int g_ring_chunk_kernel;

struct PrefillArgs {
  const __nv_bfloat16* q;          // [Tq, 16, 128] rows, row stride q_stride (elements)
  long long q_stride;
  long long q_rows;                // Tq
  const __nv_bfloat16* k;          // [Tk, 8, 128] new key rows, row stride kv_stride
  const __nv_bfloat16* v;
  long long kv_stride;
  long long kv_rows;               // Tk
  const int32_t* cu_q;             // [num_seqs + 1] query row offsets
  const int32_t* cu_k;             // [num_seqs + 1] new key row offsets (N_i >= R_i)
  int num_seqs;
  int max_seqlen_q;
  const int32_t* prefix_lens;      // [num_seqs] keys already in the seat's pages ahead of the new ones, or nullptr
  const int32_t* seat_ids;         // [num_seqs] block-table row per sequence, or nullptr (row i)
  __nv_bfloat16* k_pool;           // [num_pages, page_size, 8, 128] (needed with a prefix or write_kv)
  __nv_bfloat16* v_pool;
  int num_pages;
  int page_size;
  const int32_t* block_table;
  long long bt_stride;
  int max_pages;
  int write_kv;                    // write the new K/V rows into the pages at prefix_len + r
  int causal;
  float scale_log2;
  __nv_bfloat16* out;              // [Tq, 16, 128] rows, row stride out_stride
  long long out_stride;
  uint32_t* status;
};

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream);
// The warp-specialised TMA kernel (prefill_tma.cu); *launched = false when the call does not fit it.
cudaError_t launch_prefill_tma(const PrefillArgs& a, cudaStream_t stream, bool* launched);
// Which prefill kernel q3_prefill uses: 0 = the warp-specialised TMA kernel where the call fits it (default), 1 = the
// single-warpgroup kernel always.
extern int g_prefill_kernel;

// Host-side helpers of capi.cu shared with the allocation-free decode entry (decode_noalloc.cu).
int record_cuda_error(cudaError_t e);   // keeps the error text for q3_last_cuda_error(); returns Q3_ERR_CUDA
// The argument checks of q3_paged_decode that need no CUDA call.
int paged_decode_check_args(const void* q, int64_t q_batch_stride, const void* k_new, const void* v_new,
                            int64_t kv_new_batch_stride, const void* k_pool, const void* v_pool, int32_t num_pages,
                            int32_t page_size, const int32_t* cache_seqlens, const int32_t* block_table,
                            int64_t block_table_stride, int32_t max_pages_per_seat, int32_t batch, int32_t num_heads,
                            int32_t num_kv_heads, int32_t head_dim, const void* out, int64_t out_batch_stride,
                            int32_t num_splits);
// q3_paged_decode that also zeroes the call's ticket counters on the stream, after every check passed, before launch.
int paged_decode_clearing_counters(const void* q, int64_t q_batch_stride, const void* k_new, const void* v_new,
                                   int64_t kv_new_batch_stride, void* k_pool, void* v_pool, int32_t num_pages,
                                   int32_t page_size, const int32_t* cache_seqlens, const int32_t* block_table,
                                   int64_t block_table_stride, int32_t max_pages_per_seat, int32_t batch,
                                   int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, float softmax_scale,
                                   void* out, int64_t out_batch_stride, void* workspace, size_t workspace_bytes,
                                   int32_t num_splits, void* stream);

}  // namespace q3
