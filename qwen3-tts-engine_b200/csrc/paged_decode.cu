// Paged decode attention for the talker (one query token per seat, GQA 16/8, head_dim 128), sm_100a.
//
// Replaces flash_attn_with_kvcache(q, k_cache, v_cache, [k, v,] cache_seqlens, block_table, softmax_scale, causal)
// as called at engine/talker.py:77 (and the index_copy_ append before it, engine/talker.py:72-73, when k/v are given).
//
// Work distribution ("flat split-K"): every seat's tokens are cut into chunks of ROWS tokens; the chunks of all seats
// form one global list (seat order), and CTA c of G takes the contiguous range [c*N/G, (c+1)*N/G). Every CTA therefore
// streams the same number of K/V bytes whatever the per-seat context lengths, and the grid depends only on the batch
// bucket (graph-capturable; the split is derived on the device from cache_seqlens). A seat that straddles CTAs leaves
// one fp32 partial (o, running max, running sum) per CTA; the last CTA to finish a (seat, KV head) -- decided by an
// atomic ticket, never by waiting -- merges them. A seat inside one CTA is written directly.
//
// Inside a CTA: warp 8 (one lane) is the producer. It walks the CTA's chunk range and issues one-dimensional TMA bulk
// copies (cp.async.bulk) of whole token rows -- a row is the 2 KB of all 8 KV heads -- from the pages named by the
// block table into a ring of NSTAGES shared-memory stages, completion counted on an mbarrier per stage. Warps 0..7 are
// consumers, one per KV head: each lane owns 4 of the 128 dims for both q heads of the group, computes the partial dot
// products for every row of the chunk, and a transpose-reduction across the warp leaves one full score per lane;
// online softmax (exp2 domain) and the P.V accumulation follow in fp32.
//
// Fused append (k/v given): the new token goes at position cache_seqlens[b]; the producer copies it from k_new/v_new
// into its row of the stage, and the consumer warp of each KV head writes that row into the page pool. Only the CTA
// that owns the chunk holding the new token reads that row in this launch, so no other CTA can race with the write.
#include "q3_common.cuh"
#include "q3_kernels.h"

namespace q3 {

constexpr int kConsumerWarps = kKvHeads;           // one warp per KV head
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;

template <int ROWS, int NSTAGES>
struct DecodeSmemLayout {
  static constexpr int kStageBytes = ROWS * kRowBytes;                  // K (or V) of one chunk
  static constexpr int kKOff = 0;
  static constexpr int kVOff = NSTAGES * kStageBytes;
  static constexpr int kBarOff = 2 * NSTAGES * kStageBytes;             // full[NSTAGES], empty[NSTAGES]
  static constexpr int kPOff = kBarOff + 2 * NSTAGES * 8;               // per-warp probability buffer
  static constexpr int kMiscOff = kPOff + kConsumerWarps * 2 * ROWS * 4;
  static constexpr int kBytes = kMiscOff + 64 * 4;
};

struct SeatCursor {
  int seat;          // current seat
  long long first;   // global index of the seat's chunk 0
  int len;           // tokens the seat attends (cache + appended)
  int nch;           // chunks of the seat
};

template <int ROWS>
__device__ __forceinline__ int seat_tokens(const DecodeArgs& a, int s) {
  int L = a.seqlens[s] + (a.k_new != nullptr ? 1 : 0);
  const int cap = a.max_pages * a.page_size;
  L = L < 0 ? 0 : (L > cap ? cap : L);
  return L;
}

template <int ROWS>
__device__ __forceinline__ void advance(const DecodeArgs& a, SeatCursor& cur, long long i) {
  while (i >= cur.first + cur.nch) {
    cur.first += cur.nch;
    ++cur.seat;
    cur.len = seat_tokens<ROWS>(a, cur.seat);
    cur.nch = (cur.len + ROWS - 1) / ROWS;
  }
}

// CTA index owning global chunk p when N chunks are split over G CTAs as [c*N/G, (c+1)*N/G).
__device__ __forceinline__ int cta_of_chunk(long long p, long long N, int G) {
  return static_cast<int>(((p + 1) * G + N - 1) / N - 1);
}

__device__ __forceinline__ const __nv_bfloat16* pool_row(const __nv_bfloat16* pool, const DecodeArgs& a, int seat,
                                                         int tok, int& n_in_page) {
  const int pidx = tok / a.page_size;
  const int off = tok - pidx * a.page_size;
  int pg = a.block_table[static_cast<long long>(seat) * a.bt_stride + pidx];
  if (pg < 0 || pg >= a.num_pages) {
    atomicOr(a.status, kStatusBadPage);
    pg = 0;
  }
  n_in_page = a.page_size - off;
  return pool + (static_cast<long long>(pg) * a.page_size + off) * (kRowBytes / 2);
}

template <int ROWS, int NSTAGES, int MIN_CTAS>
__global__ void __launch_bounds__(kDecodeThreads, MIN_CTAS) paged_decode_kernel(const DecodeArgs a) {
  using SL = DecodeSmemLayout<ROWS, NSTAGES>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL::kBarOff);
  uint64_t* empty = full + NSTAGES;
  float* pbuf_all = reinterpret_cast<float*>(smem + SL::kPOff);
  volatile int* abort_flag = reinterpret_cast<int*>(smem + SL::kMiscOff);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;   // G: launched CTAs (the split is re-derived below from N)
  const bool append = a.k_new != nullptr;

  if (tid == 0) {
    for (int s = 0; s < NSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }

  // ---- plan: total chunk count N, then the seat holding this CTA's first chunk.
  long long local = 0;
  for (int s = tid; s < a.B; s += kDecodeThreads) {
    const int L = seat_tokens<ROWS>(a, s);
    local += (L + ROWS - 1) / ROWS;
    if (c == 0) {
      const int raw = a.seqlens[s] + (append ? 1 : 0);
      if (raw > a.max_pages * a.page_size || a.seqlens[s] < 0) atomicOr(a.status, kStatusBadLength);
    }
    if (L == 0 && (s % G) == c) {   // empty cache, nothing appended: the output is zero (as flash-attn writes)
      uint4* o = reinterpret_cast<uint4*>(a.out + static_cast<long long>(s) * a.out_stride);
      for (int k = 0; k < kQHeads * kHeadDim / 8; ++k) o[k] = make_uint4(0, 0, 0, 0);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
  __shared__ long long warp_sums[kConsumerWarps + 1];
  if (lane == 0) warp_sums[warp] = local;
  __syncthreads();
  long long N = 0;
#pragma unroll
  for (int w = 0; w <= kConsumerWarps; ++w) N += warp_sums[w];
  // Effective CTA count: never more CTAs than chunks, so every CTA in [0, Ge) owns at least one chunk and the
  // CTAs between a seat's first and last owner all contribute a partial (the merge counts them).
  const int Ge = static_cast<int>(N < G ? N : G);
  if (c >= Ge) return;    // uniform across the CTA; no barrier has been armed
  const long long c0 = (N * c) / Ge, c1 = (N * (c + 1)) / Ge;

  __shared__ long long plan_first;
  __shared__ int plan_seat;
  {
    long long base = 0;
    for (int t0 = 0; t0 < a.B; t0 += kDecodeThreads) {
      const int s = t0 + tid;
      const int n = s < a.B ? (seat_tokens<ROWS>(a, s) + ROWS - 1) / ROWS : 0;
      // block inclusive scan of n
      long long incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      __syncthreads();
      if (lane == 31) warp_sums[warp] = incl;
      __syncthreads();
      long long before = 0, total = 0;
#pragma unroll
      for (int w = 0; w <= kConsumerWarps; ++w) {
        if (w < warp) before += warp_sums[w];
        total += warp_sums[w];
      }
      incl += before;
      const long long excl = incl - n;
      if (n > 0 && base + excl <= c0 && c0 < base + incl) {
        plan_seat = s;
        plan_first = base + excl;
      }
      base += total;
      __syncthreads();
      if (base > c0) break;   // uniform: every thread sees the same base
    }
  }
  __syncthreads();

  SeatCursor cur;
  cur.seat = plan_seat;
  cur.first = plan_first;
  cur.len = seat_tokens<ROWS>(a, cur.seat);
  cur.nch = (cur.len + ROWS - 1) / ROWS;

  if (warp == kConsumerWarps) {
    // ================= producer
    if (lane == 0) {
      int it = 0;
      for (long long i = c0; i < c1; ++i, ++it) {
        advance<ROWS>(a, cur, i);
        const int stage = it % NSTAGES;
        if (it >= NSTAGES) {
          if (!mbar_wait_bounded(&empty[stage], ((it / NSTAGES) - 1) & 1)) {
            atomicOr(a.status, kStatusWaitTimeout);
            *abort_flag = 1;
            break;
          }
        }
        const int tok0 = static_cast<int>(i - cur.first) * ROWS;
        const int rows = min(ROWS, cur.len - tok0);
        const bool has_new = append && (tok0 + rows == cur.len);
        const int pool_rows = has_new ? rows - 1 : rows;
        uint8_t* ks = smem + SL::kKOff + stage * SL::kStageBytes;
        uint8_t* vs = smem + SL::kVOff + stage * SL::kStageBytes;
        mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(2 * rows * kRowBytes));
        for (int t = tok0; t < tok0 + pool_rows;) {
          int room;
          const __nv_bfloat16* srck = pool_row(a.k_pool, a, cur.seat, t, room);
          const __nv_bfloat16* srcv = pool_row(a.v_pool, a, cur.seat, t, room);
          const int n = min(room, tok0 + pool_rows - t);
          bulk_g2s(ks + (t - tok0) * kRowBytes, srck, n * kRowBytes, &full[stage]);
          bulk_g2s(vs + (t - tok0) * kRowBytes, srcv, n * kRowBytes, &full[stage]);
          t += n;
        }
        if (has_new) {
          const long long off = static_cast<long long>(cur.seat) * a.kv_new_stride;
          bulk_g2s(ks + (rows - 1) * kRowBytes, a.k_new + off, kRowBytes, &full[stage]);
          bulk_g2s(vs + (rows - 1) * kRowBytes, a.v_new + off, kRowBytes, &full[stage]);
        }
      }
    }
    return;
  }

  // ================= consumers: warp h = KV head h, q heads 2h and 2h+1
  const int h = warp;
  float* pbuf = pbuf_all + warp * 2 * ROWS;
  constexpr int NV = 2 * ROWS;
  constexpr int kDupShift = (NV == 32) ? 0 : (NV == 16 ? 1 : (NV == 8 ? 2 : 3));   // lanes sharing one value
  const int my_idx = lane >> kDupShift;           // value index held after the transpose-reduction
  const int my_g = my_idx / ROWS;                 // q head within the group (== lane >> 4)
  const int my_r = my_idx % ROWS;                 // row within the chunk
  const bool my_owner = (lane & ((1 << kDupShift) - 1)) == 0;

  float4 q0 = make_float4(0, 0, 0, 0), q1 = q0, o0 = q0, o1 = q0;
  float m0 = -INFINITY, m1 = -INFINITY, lsum = 0.f;
  int it = 0;
  int seat_started = -1;
  for (long long i = c0; i < c1; ++i, ++it) {
    advance<ROWS>(a, cur, i);
    if (cur.seat != seat_started) {   // first chunk of a seat within this CTA: load q, reset the running state
      seat_started = cur.seat;
      const __nv_bfloat16* qp = a.q + static_cast<long long>(cur.seat) * a.q_stride + (2 * h) * kHeadDim + 4 * lane;
      q0 = bf16x4_to_float4(ld_nc_u2(qp));
      q1 = bf16x4_to_float4(ld_nc_u2(qp + kHeadDim));
      q0.x *= a.scale_log2; q0.y *= a.scale_log2; q0.z *= a.scale_log2; q0.w *= a.scale_log2;
      q1.x *= a.scale_log2; q1.y *= a.scale_log2; q1.z *= a.scale_log2; q1.w *= a.scale_log2;
      o0 = make_float4(0, 0, 0, 0);
      o1 = o0;
      m0 = m1 = -INFINITY;
      lsum = 0.f;
    }
    const int stage = it % NSTAGES;
    if (!mbar_wait_bounded(&full[stage], (it / NSTAGES) & 1)) {
      atomicOr(a.status, kStatusWaitTimeout);
      *abort_flag = 1;
      break;
    }
    const int jchunk = static_cast<int>(i - cur.first);
    const int tok0 = jchunk * ROWS;
    const int rows = min(ROWS, cur.len - tok0);
    const uint8_t* kb = smem + SL::kKOff + stage * SL::kStageBytes + h * kHeadBytes + lane * 8;
    const uint8_t* vb = smem + SL::kVOff + stage * SL::kStageBytes + h * kHeadBytes + lane * 8;

    // ---- scores
    float s[NV];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      if (r < rows) {
        const float4 k = bf16x4_to_float4(*reinterpret_cast<const uint2*>(kb + r * kRowBytes));
        s[r] = q0.x * k.x + q0.y * k.y + q0.z * k.z + q0.w * k.w;
        s[ROWS + r] = q1.x * k.x + q1.y * k.y + q1.z * k.z + q1.w * k.w;
      } else {
        s[r] = 0.f;
        s[ROWS + r] = 0.f;
      }
    }
    const float sc = transpose_reduce<NV>(s, lane);
    const bool valid = my_r < rows;
    const float x = valid ? sc : -INFINITY;
    float cm = x;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    const float cm0 = __shfl_sync(0xffffffffu, cm, 0);
    const float cm1 = __shfl_sync(0xffffffffu, cm, 16);
    const float mn0 = fmaxf(m0, cm0), mn1 = fmaxf(m1, cm1);
    const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    const float p = valid ? exp2f(x - (my_g ? mn1 : mn0)) : 0.f;
    lsum = lsum * (my_g ? a1 : a0) + (my_owner ? p : 0.f);
    if (my_owner) pbuf[my_idx] = p;
    o0.x *= a0; o0.y *= a0; o0.z *= a0; o0.w *= a0;
    o1.x *= a1; o1.y *= a1; o1.z *= a1; o1.w *= a1;
    __syncwarp();

    // ---- P.V
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      if (r < rows) {
        const float p0 = pbuf[r], p1 = pbuf[ROWS + r];
        const float4 v = bf16x4_to_float4(*reinterpret_cast<const uint2*>(vb + r * kRowBytes));
        o0.x += p0 * v.x; o0.y += p0 * v.y; o0.z += p0 * v.z; o0.w += p0 * v.w;
        o1.x += p1 * v.x; o1.y += p1 * v.y; o1.z += p1 * v.z; o1.w += p1 * v.w;
      }
    }

    // ---- fused append: this chunk holds the new token; write its head-h row into the pools
    if (append && tok0 + rows == cur.len) {
      int room;
      const int t = cur.len - 1;
      __nv_bfloat16* dk = const_cast<__nv_bfloat16*>(pool_row(a.k_pool, a, cur.seat, t, room));
      __nv_bfloat16* dv = const_cast<__nv_bfloat16*>(pool_row(a.v_pool, a, cur.seat, t, room));
      *reinterpret_cast<uint2*>(dk + h * kHeadDim + 4 * lane) =
          *reinterpret_cast<const uint2*>(kb + (rows - 1) * kRowBytes);
      *reinterpret_cast<uint2*>(dv + h * kHeadDim + 4 * lane) =
          *reinterpret_cast<const uint2*>(vb + (rows - 1) * kRowBytes);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);

    // ---- end of the seat's chunks in this CTA
    const bool seat_done = (jchunk == cur.nch - 1) || (i == c1 - 1);
    if (seat_done) {
      float lg = lsum;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) lg += __shfl_xor_sync(0xffffffffu, lg, o);
      const float l0 = __shfl_sync(0xffffffffu, lg, 0);
      const float l1 = __shfl_sync(0xffffffffu, lg, 16);
      const int c_first = cta_of_chunk(cur.first, N, Ge);
      const int c_last = cta_of_chunk(cur.first + cur.nch - 1, N, Ge);
      __nv_bfloat16* op = a.out + static_cast<long long>(cur.seat) * a.out_stride + (2 * h) * kHeadDim + 4 * lane;
      if (c_first == c_last) {
        const float r0 = 1.f / l0, r1 = 1.f / l1;
        *reinterpret_cast<uint2*>(op) = float4_to_bf16x4(make_float4(o0.x * r0, o0.y * r0, o0.z * r0, o0.w * r0));
        *reinterpret_cast<uint2*>(op + kHeadDim) =
            float4_to_bf16x4(make_float4(o1.x * r1, o1.y * r1, o1.z * r1, o1.w * r1));
      } else {
        const long long slot = static_cast<long long>(c) + cur.seat;
        float* wo = a.ws_o + ((slot * kKvHeads + h) * kGroup) * kHeadDim;
        float* wml = a.ws_ml + ((slot * kKvHeads + h) * kGroup) * 2;
        reinterpret_cast<float4*>(wo)[lane] = o0;
        reinterpret_cast<float4*>(wo + kHeadDim)[lane] = o1;
        if (lane == 0) {
          wml[0] = m0; wml[1] = l0; wml[2] = m1; wml[3] = l1;
        }
        __threadfence();
        __syncwarp();
        unsigned ticket = 0;
        if (lane == 0) ticket = atomicAdd(a.counters + static_cast<long long>(cur.seat) * kKvHeads + h, 1u);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket == static_cast<unsigned>(c_last - c_first)) {
          // last partial of this (seat, KV head): merge all of them in CTA order
          __threadfence();
          float M0 = -INFINITY, M1 = -INFINITY;
          for (int cc = c_first; cc <= c_last; ++cc) {
            const float* ml = a.ws_ml + (((static_cast<long long>(cc) + cur.seat) * kKvHeads + h) * kGroup) * 2;
            M0 = fmaxf(M0, __ldcg(ml + 0));
            M1 = fmaxf(M1, __ldcg(ml + 2));
          }
          float4 O0 = make_float4(0, 0, 0, 0), O1 = O0;
          float L0 = 0.f, L1 = 0.f;
          for (int cc = c_first; cc <= c_last; ++cc) {
            const long long sl = static_cast<long long>(cc) + cur.seat;
            const float* ml = a.ws_ml + ((sl * kKvHeads + h) * kGroup) * 2;
            const float* po = a.ws_o + ((sl * kKvHeads + h) * kGroup) * kHeadDim;
            const float w0 = exp2f(__ldcg(ml + 0) - M0), w1 = exp2f(__ldcg(ml + 2) - M1);
            L0 += __ldcg(ml + 1) * w0;
            L1 += __ldcg(ml + 3) * w1;
            const float4 x0 = __ldcg(reinterpret_cast<const float4*>(po) + lane);
            const float4 x1 = __ldcg(reinterpret_cast<const float4*>(po + kHeadDim) + lane);
            O0.x += x0.x * w0; O0.y += x0.y * w0; O0.z += x0.z * w0; O0.w += x0.w * w0;
            O1.x += x1.x * w1; O1.y += x1.y * w1; O1.z += x1.z * w1; O1.w += x1.w * w1;
          }
          const float r0 = 1.f / L0, r1 = 1.f / L1;
          *reinterpret_cast<uint2*>(op) = float4_to_bf16x4(make_float4(O0.x * r0, O0.y * r0, O0.z * r0, O0.w * r0));
          *reinterpret_cast<uint2*>(op + kHeadDim) =
              float4_to_bf16x4(make_float4(O1.x * r1, O1.y * r1, O1.z * r1, O1.w * r1));
          if (lane == 0) a.counters[static_cast<long long>(cur.seat) * kKvHeads + h] = 0u;   // ready for the next launch
        }
      }
    }
    if (*abort_flag) break;
  }
}

// ------------------------------------------------------------------ host-side launch
template <int ROWS, int NSTAGES, int MIN_CTAS>
static cudaError_t launch_decode(const DecodeArgs& a, int grid, cudaStream_t stream) {
  using SL = DecodeSmemLayout<ROWS, NSTAGES>;
  auto kern = paged_decode_kernel<ROWS, NSTAGES, MIN_CTAS>;
  static thread_local int configured_device = -1;   // attribute set once per (thread, device), before any capture
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SL::kBytes);
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  kern<<<grid, kDecodeThreads, SL::kBytes, stream>>>(a);
  return cudaGetLastError();
}

int decode_rows_per_chunk(int variant) { return variant == 1 ? 8 : 16; }

int decode_ctas_per_sm(int variant) { return variant == 1 ? 2 : 1; }

cudaError_t launch_paged_decode(const DecodeArgs& a, int grid, int variant, cudaStream_t stream) {
  switch (variant) {
    case 1: return launch_decode<8, 3, 2>(a, grid, stream);    // 96 KB: two CTAs per SM
    case 2: return launch_decode<16, 2, 1>(a, grid, stream);   // 128 KB
    default: return launch_decode<16, 3, 1>(a, grid, stream);  // 192 KB: one CTA per SM
  }
}

}  // namespace q3
