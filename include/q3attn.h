/* q3attn — B200 (sm_100a) attention hot path of a Qwen3-TTS streaming engine, as a C ABI.
 *
 * Every entry point takes raw device pointers, element strides and sizes, launches on the given CUDA stream
 * (a cudaStream_t passed as void*, NULL = the legacy default stream) and returns Q3_OK or an error code. Nothing here
 * allocates, synchronises or reads device memory on the host, so every call can be recorded inside a CUDA graph
 * (make the first call of each entry point on a device outside capture: it sets kernel attributes).
 *
 * Tensor conventions (the engine's model family: 16 query heads, 8 KV heads, head_dim 128, bf16 storage):
 *   q rows          [B, 16, 128]        innermost 128 contiguous, heads contiguous; batch stride given
 *   K/V page pool   [num_pages, page_size, 8, 128] fully contiguous (one token row = 2048 bytes)
 *   block table     int32 [B, stride]   physical page of each seat's j-th page
 *   code-predictor  K/V [B, 8, S, 128]  (S >= n_live) with explicit batch/head/slot strides
 * Only num_heads=16, num_kv_heads=8, head_dim=128 are compiled; other shapes return Q3_ERR_UNSUPPORTED.
 *
 * Each function names the reference interface (saicherry93479/Qwen3-TTS-Engine, path:line) it replaces.
 */
#ifndef Q3ATTN_H_
#define Q3ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q3_OK 0
#define Q3_ERR_INVALID 1      /* null pointer, negative size, inconsistent strides */
#define Q3_ERR_UNSUPPORTED 2  /* head counts / head_dim / slot count outside the compiled family */
#define Q3_ERR_ALIGNMENT 3    /* a pointer or stride breaks the 16-byte (pools, new rows, decode q) or 8-byte rule */
#define Q3_ERR_WORKSPACE 4    /* workspace missing or smaller than q3_paged_decode_workspace_bytes() */
#define Q3_ERR_CUDA 5         /* a CUDA runtime call failed; see q3_last_cuda_error() */
#define Q3_ERR_SCRATCH_LIMIT 6  /* q3_paged_decode_noalloc: batch / split count beyond its fixed 16 MiB scratch */

/* Status bits a kernel may set on the device (read with q3_read_status). */
#define Q3_STATUS_WAIT_TIMEOUT 1u  /* a pipeline wait gave up (kernel returned early; outputs invalid) */
#define Q3_STATUS_BAD_PAGE 2u      /* a block-table entry or slot outside the pool (access skipped / clamped) */
#define Q3_STATUS_BAD_LENGTH 4u    /* a sequence length beyond the seat's block-table capacity (clamped) */

int q3_version(void);
const char* q3_error_string(int code);
/* Text of the last CUDA error seen by this thread's q3 calls ("" if none). */
const char* q3_last_cuda_error(void);
/* Streaming multiprocessors of the current device (148 on B200). */
int q3_device_sm_count(void);
/* Read (and optionally clear) the device status word of the current device. Synchronous; not for the hot loop. */
int q3_read_status(uint32_t* status_out, int clear);
/* Self-test of the failure reporting every pipeline kernel shares: launches one kernel whose bounded wait (on an
 * mbarrier nothing arrives on) expires after limit_ns (1 .. 100,000,000 ns), which raises Q3_STATUS_WAIT_TIMEOUT and
 * returns; the context stays usable. Asynchronous on `stream`. No reference counterpart (the reference has no
 * device-side waits). */
int q3_selftest_bounded_wait(uint64_t limit_ns, void* stream);

/* ---------------------------------------------------------------- paged decode attention
 * Replaces flash_attn_with_kvcache(q, k_cache, v_cache, k=, v=, cache_seqlens=, block_table=, softmax_scale=,
 * causal=True) as called at engine/talker.py:77, and, when k_new/v_new are given, the index_copy_ append before it
 * (engine/talker.py:72-73) fused into the same launch.
 *   k_new == NULL: seat b attends over cache_seqlens[b] tokens.
 *   k_new != NULL: the new K/V row of seat b is written at position cache_seqlens[b] and seat b attends over
 *                  cache_seqlens[b] + 1 tokens (flash-attn's k/v-append semantics).
 * A seat with nothing to attend gets a zero output. num_splits = CTAs sharing the work (0 = SMs x resident CTAs).
 * The workspace (q3_paged_decode_workspace_bytes) must be zero-filled once before its first use; every launch leaves
 * it ready for the next. Calls that share one workspace must not overlap on the GPU. */
size_t q3_paged_decode_workspace_bytes(int32_t batch, int32_t num_splits);
int q3_paged_decode(const void* q, int64_t q_batch_stride,
                    const void* k_new, const void* v_new, int64_t kv_new_batch_stride,
                    void* k_pool, void* v_pool, int32_t num_pages, int32_t page_size,
                    const int32_t* cache_seqlens,
                    const int32_t* block_table, int64_t block_table_stride, int32_t max_pages_per_seat,
                    int32_t batch, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                    float softmax_scale,
                    void* out, int64_t out_batch_stride,
                    void* workspace, size_t workspace_bytes, int32_t num_splits,
                    void* stream);
/* Kernel variant used by q3_paged_decode: 0 = 8-token chunks x 3 stages, two CTAs per SM,
 * 1 = 16-token chunks x 3 stages, one CTA per SM, 2 = 8-token chunks x 2 stages, two CTAs per SM,
 * 3 / 4 = warp-MMA scoring (mma.sync) with early stage release, 8-token chunks x 3 / 2 stages, two CTAs per SM,
 * 5 = dedicated producer warps: one 20-warp CTA per SM running two 8-token x 3-stage chunk streams (default).
 * Values outside 0..5 leave the selection unchanged. Returns the previous value. No reference counterpart (a tuning
 * knob of this library). */
int q3_set_decode_variant(int variant);
/* CTAs of the given decode variant that the runtime can keep resident on one SM of the current device. */
int q3_paged_decode_resident_ctas(int variant);

/* Same as q3_paged_decode, for callers that cannot allocate device memory (no workspace argument). No counterpart in
 * the reference: it exists for hosts whose device memory comes from an arena they do not own, or whose calls must not
 * allocate. The split-K scratch lives in a 16 MiB array compiled into the library, held by every GPU that loads it
 * until exit; calls whose workspace would exceed it (roughly batch + CTAs > 2000) return Q3_ERR_SCRATCH_LIMIT before
 * launching anything. The first call on a device looks up the array's device address (do it before any stream
 * capture); the address is cached per device, so after a cudaDeviceReset the library must be reloaded. Arguments are
 * checked before anything is queued: a refused call leaves the array alone. Every accepted call clears the counters it
 * uses on its stream; calls that overlap on the GPU share the array and race. */
int q3_paged_decode_noalloc(const void* q, int64_t q_batch_stride,
                            const void* k_new, const void* v_new, int64_t kv_new_batch_stride,
                            void* k_pool, void* v_pool, int32_t num_pages, int32_t page_size,
                            const int32_t* cache_seqlens,
                            const int32_t* block_table, int64_t block_table_stride, int32_t max_pages_per_seat,
                            int32_t batch, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                            float softmax_scale,
                            void* out, int64_t out_batch_stride, int32_t num_splits,
                            void* stream);

/* ---------------------------------------------------------------- K/V append into pages
 * Replaces kc[l].view(-1, nkv, hd).index_copy_(0, slot, k) (and the same for V): engine/talker.py:72-73 and 161-162,
 * engine/arrivals.py:144-145. Row i of k/v (n_rows rows of num_kv_heads*head_dim bf16, row stride row_stride
 * elements) is written to pool row slots[i] (flat row index in [0, pool_rows)). Placement is bit-exact. */
int q3_kv_append_slots(const void* k, const void* v, int64_t row_stride,
                       void* k_pool, void* v_pool, int64_t pool_rows,
                       int32_t num_kv_heads, int32_t head_dim,
                       const int64_t* slots, int32_t n_rows, void* stream);
/* Same, addressed by (seat, position) through the block table: row i goes to token positions[i] of seat
 * seat_of_row[i] (seat_of_row == NULL: seat i), i.e. pool row block_table[seat, pos / page_size] * page_size +
 * pos % page_size. */
int q3_kv_append_paged(const void* k, const void* v, int64_t row_stride,
                       void* k_pool, void* v_pool, int32_t num_pages, int32_t page_size,
                       int32_t num_kv_heads, int32_t head_dim,
                       const int32_t* positions, const int32_t* seat_of_row,
                       const int32_t* block_table, int64_t block_table_stride, int32_t max_pages_per_seat,
                       int32_t n_rows, void* stream);

/* ---------------------------------------------------------------- prefill attention (tcgen05 tensor cores)
 * Replaces flash_attn_varlen_func(q, k, v, cu, cu, max, max, softmax_scale, causal=True) (engine/talker.py:169) and
 * flash_attn_func(q, K, V, softmax_scale, causal=True) over a cached prefix (engine/arrivals.py:148), and fuses the
 * page writes of engine/talker.py:161-162 / engine/arrivals.py:144-145 when write_kv is set.
 * Sequence i: query rows [cu_seqlens_q[i], cu_seqlens_q[i+1]) (R_i), new key rows [cu_seqlens_k[i], cu_seqlens_k[i+1])
 * (N_i >= R_i) of k/v [Tk, 8, 128], and prefix_lens[i] keys already in the pages of block-table row seat_ids[i]
 * (prefix_lens NULL: none; seat_ids NULL: row i). Keys are indexed prefix first; with causal, query j sees keys
 * 0 .. prefix + N - R + j (bottom-right alignment). write_kv: the new rows also go to positions prefix + r of the
 * seat's pages. max_seqlen_q must be >= every R_i; q_rows = Tq and kv_rows = Tk are the row counts of q and k/v (no
 * row at or past them is read). Output rows [Tq, 16, 128] bf16. */
int q3_prefill(const void* q, int64_t q_row_stride, int64_t q_rows,
               const void* k, const void* v, int64_t kv_row_stride, int64_t kv_rows,
               const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t num_seqs, int32_t max_seqlen_q,
               const int32_t* prefix_lens, const int32_t* seat_ids,
               void* k_pool, void* v_pool, int32_t num_pages, int32_t page_size,
               const int32_t* block_table, int64_t block_table_stride, int32_t max_pages_per_seat,
               int32_t write_kv, int32_t causal, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
               float softmax_scale, void* out, int64_t out_row_stride, void* stream);

/* Prefill kernel used by q3_prefill: 0 = the warp-specialised TMA kernel wherever the call fits it (default; other
 * calls use kernel 1), 1 = the single-warpgroup kernel for every call. Other values leave the selection unchanged.
 * Returns the previous value. No reference counterpart (a tuning knob of this library). */
int q3_set_prefill_kernel(int kernel);

/* ---------------------------------------------------------------- code-predictor attention
 * Replaces cp_attn(q, K, V, n_live, scale) (engine/cp_attn.py:33-39), i.e. the attention expression of
 * CodePredictor._post (engine/code_predictor.py:46-47): q [B,16,128] over slots 0..n_live-1 of K/V [B,8,S,128];
 * fp32 scores, softmax, probabilities and P.V, bf16 out [B, 2048]. 1 <= n_live <= min(S,16). */
int q3_cp_attn(const void* q, int64_t q_batch_stride,
               const void* K, const void* V,
               int64_t k_batch_stride, int64_t k_head_stride, int64_t k_slot_stride,
               int64_t v_batch_stride, int64_t v_head_stride, int64_t v_slot_stride,
               int32_t batch, int32_t n_slots, int32_t n_live, float softmax_scale,
               void* out, int64_t out_batch_stride, void* stream);
/* One fused code-predictor step: writes k_new/v_new [B,8,128] into slot `slot` of K/V (engine/code_predictor.py:58,
 * K.index_copy_(2, [p], k)) and attends over slots 0..slot (n_live = slot + 1), one launch per (step, layer). */
int q3_cp_step(const void* q, int64_t q_batch_stride,
               const void* k_new, const void* v_new, int64_t kv_new_batch_stride,
               void* K, void* V,
               int64_t k_batch_stride, int64_t k_head_stride, int64_t k_slot_stride,
               int64_t v_batch_stride, int64_t v_head_stride, int64_t v_slot_stride,
               int32_t batch, int32_t n_slots, int32_t slot, float softmax_scale,
               void* out, int64_t out_batch_stride, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Attention layers from the QKV projection, with the q/k RMSNorm and rotate-half RoPE of engine/ops.py:51-60 fused
 * into the attention kernels (bf16 rounding points of the reference's eager source: normalise in fp32 and round,
 * times the weight and round, x*cos and rot(x)*sin each rounded, their sum rounded).
 * qkv rows are [q (16x128) | k (8x128) | v (8x128)] bf16, qkv_row_stride elements apart (16-byte aligned rows). */
typedef struct q3_qk_norm_rope {
  const void* q_norm_weight;   /* [128] bf16 (w.qn) */
  const void* k_norm_weight;   /* [128] bf16 (w.kn) */
  const void* cos;             /* [rows, 128] bf16: row b serves batch row b ... */
  const void* sin;
  int64_t rope_row_stride;     /* ... rows rope_row_stride elements apart; 0 = one row for every batch row */
  float eps;                   /* 1e-6 in the reference (ops.py:51) */
} q3_qk_norm_rope;

/* One talker attention layer after the QKV GEMM: engine/talker.py:69-77 (q = rope(rms(q, qn)), k = rope(rms(k, kn)),
 * the k/v index_copy_ into the pools at position cache_seqlens[b], flash_attn_with_kvcache over cache + new row).
 * cos/sin row b must be the rotary row of position cache_seqlens[b] (W.cos[pos], talker.py:111). Pools, table,
 * workspace (q3_paged_decode_workspace_bytes) and errors as q3_paged_decode; the kernel of q3_set_decode_variant 5 (the
 * default) when that is selected, else that of variant 0. */
int q3_paged_decode_qkv(const void* qkv, int64_t qkv_row_stride, const q3_qk_norm_rope* norm_rope,
                        void* k_pool, void* v_pool, int32_t num_pages, int32_t page_size,
                        const int32_t* cache_seqlens,
                        const int32_t* block_table, int64_t block_table_stride, int32_t max_pages_per_seat,
                        int32_t batch, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                        float softmax_scale,
                        void* out, int64_t out_batch_stride,
                        void* workspace, size_t workspace_bytes, int32_t num_splits,
                        void* stream);
/* One code-predictor (step, layer) after the QKV GEMM: engine/code_predictor.py:40-41 (q/k norm + RoPE with
 * cp_cos/cp_sin[p]), :58 (slot-p write) and :46-47 (attention over slots 0..p), in one launch. K/V strides as
 * q3_cp_step. */
int q3_cp_step_qkv(const void* qkv, int64_t qkv_row_stride, const q3_qk_norm_rope* norm_rope,
                   void* K, void* V,
                   int64_t k_batch_stride, int64_t k_head_stride, int64_t k_slot_stride,
                   int64_t v_batch_stride, int64_t v_head_stride, int64_t v_slot_stride,
                   int32_t batch, int32_t n_slots, int32_t slot, float softmax_scale,
                   void* out, int64_t out_batch_stride, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Row kernels around the attention layers (one launch each instead of a chain of small ops), bf16 rounding points
 * of the reference's eager source. */
/* Residual add + RMSNorm (engine/ops.py:51-55 after the residual adds of talker.py:78-79 / code_predictor.py:48-50):
 * with residual given, x = bf16(x + residual) is written back to x first; then
 * out = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))). hidden 1024 or 2048; rows 16-byte aligned. */
int q3_add_rms_norm(void* x, int64_t x_row_stride, const void* residual, int64_t residual_row_stride,
                    const void* weight, void* out, int64_t out_row_stride, int64_t rows, int32_t hidden, float eps,
                    void* stream);
/* SiLU-gated product of the MLP (engine/ops.py:63-65): out = bf16(bf16(silu(g)) * u) for gate_up = [g | u]
 * [rows, 2 * ffn]. */
int q3_silu_mul(const void* gate_up, int64_t gate_up_row_stride, void* out, int64_t out_row_stride, int64_t rows,
                int32_t ffn, void* stream);
/* q/k RMSNorm + RoPE (engine/ops.py:51-60 as called at talker.py:69-70, arrivals.py:114-115) in place on QKV rows
 * [q 16x128 | k 8x128 | v 8x128]; cos/sin row r serves row r (rope_row_stride 0: one row for all). */
int q3_qk_norm_rope_rows(void* qkv, int64_t qkv_row_stride, const q3_qk_norm_rope* norm_rope, int64_t rows,
                         void* stream);

/* Windowed ring attention of the streaming codec decoder, fp16, one transformer layer (engine/decoder_stream.py:147-181,
 * ring mode). Stream b's rotated keys / values of recent frames live in a ring of `ring` slots (frame f in slot
 * f % ring) at k_ring + ring_rows[b] * ring_stream_stride + slot * ring_slot_stride + head * head_dim (elements).
 * The chunk's n frames at positions pos[b] .. pos[b]+n-1 (q / k_new / v_new [B, n, heads, head_dim] rows) attend
 * over the ring frames within `past` frames before them and over the chunk's keys up to themselves, with the
 * reference's fp16 rounding points (scores, P and each P.V half rounded to fp16). write_new != 0 also stores the
 * chunk's K/V into ring slots (pos + j) % ring (the caller's index_copy_, decoder_stream.py:330-333).
 * head_dim 64 or 128, ring <= 128, n <= min(17, ring - past). out: [B, n, heads * head_dim] fp16. */
/* One-frame ring kernel used by q3_ring_window_attn for n == 1: 6 = nothing staged, 4 (head_dim 64) or 8 (128) warps
 * per (stream, head) loading their rows straight into registers (ring >= 2, past <= 79; the default, the fastest
 * measured); 2 = scalar math, one warp per head, G heads per CTA (4 for head_dim 64, 2 for 128; also the calls with
 * wider windows under the default); 1 = scalar math, one CTA per (stream, head); 0 = tensor cores, one warp per head, G = 4 / 2,
 * 3 = G = 2 / 1, 4 = G = 1 (past < 96); 5 = a persistent TMA pipeline, quads of four warps per (stream, head) fed by
 * producer warps (head_dim 64, past <= 97). Calls a selection does not fit (G not dividing the head count, sizes) run
 * kernel 1. Other values leave the selection unchanged.
 * Returns the previous value. No reference counterpart (a tuning knob of this library). */
int q3_set_ring_frame_kernel(int kernel);
/* Kernel used by q3_ring_window_attn for chunks of 2 .. 17 frames: 1 = one CTA per (stream, head), tensor cores
 * (the default, the fastest measured; also every call another selection does not fit); 0 = tensor cores, one warp per
 * head, G heads per CTA (2 for head_dim 64, 1 for 128), 2 = G = 4 / 2, 3 = G = 1 (up to 16 frames, past + n <= 112);
 * 4 = the persistent TMA pipeline of selection 5 above for 2 .. 8 frames (head_dim 64, 66 <= past <= 97).
 * Other values leave the selection unchanged. Returns the previous value. No reference counterpart (a tuning knob of
 * this library). */
int q3_set_ring_chunk_kernel(int kernel);
int q3_ring_window_attn(const void* q, const void* k_new, const void* v_new, int64_t qkv_batch_stride,
                        int64_t qkv_frame_stride, void* k_ring, void* v_ring, int64_t ring_stream_stride,
                        int64_t ring_slot_stride, const int64_t* ring_rows, const int64_t* pos, int32_t batch,
                        int32_t n, int32_t heads, int32_t head_dim, int32_t ring, int32_t past, float scale,
                        int32_t write_new, void* out, int64_t out_batch_stride, int64_t out_frame_stride,
                        void* stream);

/* Shared-prefix copy at admission (engine/arrivals.py:67-96 keeps, per (voice, language), the K/V of the k prompt
 * positions every request of that voice shares; arrivals.py:139-145 writes them into each admitted seat). For every
 * layer l < num_layers, batch row b and prefix row r < prefix_len, the K and V rows at
 * src + l * src_layer_stride + slot[b] * src_slot_stride + r * (num_kv_heads * head_dim) (elements, 16-byte aligned)
 * land at position r of seat[b] in layer l's pools, through the block table. k_pools / v_pools are DEVICE arrays of
 * the num_layers pool base addresses (16-byte aligned, pool_rows rows each). One launch. */
int q3_kv_copy_prefix(const void* k_src, const void* v_src, int64_t src_layer_stride, int64_t src_slot_stride,
                      const uint64_t* k_pools, const uint64_t* v_pools, int32_t num_layers, int64_t pool_rows,
                      int32_t page_size, int32_t num_kv_heads, int32_t head_dim,
                      const int64_t* seat, const int64_t* slot, int32_t batch, int32_t prefix_len,
                      const int32_t* block_table, int64_t block_table_stride, int32_t max_pages_per_seat,
                      void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Logit processing + top-k / temperature sampling, one call per sampled token of a frame. Replaces
 * Talker._cb0_logits (engine/talker.py:90-94: repetition penalty over the seat's `seen` row, + suppress row, EOS masked
 * while ngen < min_new), sample_topk (engine/ops.py:68-76: topk, softmax(vals / temperature), multinomial) and the
 * embedding lookup of the sampled id (engine/code_predictor.py:68, 71). top_k = 1 is greedy (the maximum; equal maxima
 * resolve to the lowest index). The random stream is Philox4x32-10 keyed by `seed`, counter (row, launch index); the
 * launch index lives in rng_state[0] on the device and advances by one per call (CUDA-graph replays included), so
 * draws are reproducible from (seed, rng_state) but are not torch.multinomial's stream. Optional parts are switched off
 * with null pointers. */
typedef struct q3_sampler {
  const void* logits;          /* [batch, vocab] rows, row_stride elements apart */
  int32_t logits_dtype;        /* 0 = bf16, 1 = fp32 */
  int64_t row_stride;
  int32_t batch;
  int32_t vocab;               /* <= 4096 */
  int32_t top_k;               /* 1..min(64, vocab) */
  float temperature;           /* > 0 when top_k > 1 */
  const uint8_t* seen;         /* optional [*, vocab] bool rows: repetition penalty on seen ids (row = seat[b]) */
  int64_t seen_row_stride;
  const int64_t* seat;         /* [batch]: row of seen / ngen for each batch row (required with seen or ngen) */
  float repetition_penalty;
  const float* bias;           /* optional [vocab] fp32 added after the penalty (the suppress row) */
  const int64_t* ngen;         /* optional: EOS (eos_id) masked to -inf while ngen[seat[b]] < min_new */
  int32_t min_new;
  int32_t eos_id;
  uint64_t seed;
  uint64_t* rng_state;         /* device [2] uint64, zero-initialised once by the caller; one stream per state */
  int64_t* out_ids;            /* [batch] sampled ids, out_stride elements apart */
  int64_t out_stride;
  const void* emb;             /* optional [>= vocab rows, emb_dim] bf16 table: row out_ids[b] -> emb_out row b */
  int64_t emb_row_stride;
  int32_t emb_dim;
  void* emb_out;
  int64_t emb_out_row_stride;
} q3_sampler;
int q3_sample_topk(const q3_sampler* sampler, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* Q3ATTN_H_ */
