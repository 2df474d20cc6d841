// Paged decode attention for the talker (one query token per seat, GQA 16/8, head_dim 128), sm_100a.
//
// Replaces flash_attn_with_kvcache(q, k_cache, v_cache, [k, v,] cache_seqlens, block_table, softmax_scale, causal)
// as called at engine/talker.py:77 (and the index_copy_ append before it, engine/talker.py:72-73, when k/v are given).
//
// Work distribution ("flat split-K"): every seat's tokens are cut into chunks of ROWS tokens; the chunks of all seats
// form one global list (seat order), and CTA c of Ge takes the contiguous range [c*N/Ge, (c+1)*N/Ge), where N is the
// total chunk count and Ge = min(launched CTAs, N). Every CTA therefore streams the same number of K/V bytes whatever
// the per-seat context lengths, and the grid depends only on the batch bucket (graph-capturable; the split is derived
// on the device from cache_seqlens). A seat that straddles CTAs leaves one fp32 partial (o, running max, running sum)
// per CTA; the last CTA to finish a (seat, KV head) -- decided by an atomic ticket, never by waiting -- merges them.
// A seat inside one CTA is written directly.
//
// Inside a CTA there are 8 warps, one per KV head, and no dedicated producer: K and V of a chunk (ROWS token rows of
// 2 KB, all 8 heads) are brought into a ring of NSTAGES shared-memory stages by one-dimensional TMA bulk copies
// (cp.async.bulk) whose completion is counted on an mbarrier per stage. Warp 0 issues the first NSTAGES chunks; after
// that, the warp that is LAST to finish reading a stage (a shared-memory ticket per stage) refills it with the chunk
// NSTAGES further on. Keeping the CTA at 8 warps lets two CTAs share an SM at 128 registers per thread (the register
// file is split over the SM's four sub-partitions, 16K registers each).
//
// Scores: lane l of warp h scores row l / LPR of the chunk over DPL of the 128 dims, for both q heads of the group,
// with packed fp32 FMAs (FFMA2); LPR lanes per row combine with shuffles. Online softmax in the exp2 domain.
// P.V: lane l owns dims 4l..4l+3 of both q heads.
//
// Fused append (k/v given): the new token goes at position cache_seqlens[b]; its row is copied from k_new/v_new into
// the stage, and each warp writes its head's 256 bytes of that row into the page pool. Only the CTA that owns the
// chunk holding the new token reads that row in this launch, so no other CTA can race with the write.
#include "q3_common.cuh"
#include "q3_kernels.h"

namespace q3 {

constexpr int kDecodeWarps = kKvHeads;             // one warp per KV head
constexpr int kDecodeThreads = kDecodeWarps * 32;  // 256

template <int ROWS, int NSTAGES>
struct DecodeSmemLayout {
  static constexpr int kStageBytes = ROWS * kRowBytes;                  // K (or V) of one chunk
  static constexpr int kKOff = 0;
  static constexpr int kVOff = NSTAGES * kStageBytes;
  static constexpr int kBarOff = 2 * NSTAGES * kStageBytes;             // full[NSTAGES] mbarriers
  static constexpr int kDoneOff = kBarOff + NSTAGES * 8;                // done[NSTAGES] reader tickets
  static constexpr int kPOff = kDoneOff + ((NSTAGES * 4 + 15) / 16) * 16;   // per-warp probabilities [ROWS][2]
  static constexpr int kMiscOff = kPOff + kDecodeWarps * 2 * ROWS * 4;
  static constexpr int kBytes = kMiscOff + 64;
};

struct SeatCursor {
  int seat;          // current seat
  long long first;   // global index of the seat's chunk 0
  int len;           // tokens the seat attends (cache + appended)
  int nch;           // chunks of the seat
};

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
    cur.len = seat_tokens(a, cur.seat);
    cur.nch = (cur.len + ROWS - 1) / ROWS;
  }
}

__device__ __forceinline__ uint32_t word_of(const uint4& w, int e) {
  return e == 0 ? w.x : (e == 1 ? w.y : (e == 2 ? w.z : w.w));
}

__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t x) {
  return make_float2(__uint_as_float(x << 16), __uint_as_float(x & 0xffff0000u));
}

// CTA index owning global chunk p when N chunks are split over Ge CTAs as [c*N/Ge, (c+1)*N/Ge).
__device__ __forceinline__ int cta_of_chunk(long long p, long long N, int Ge) {
  return static_cast<int>(((p + 1) * Ge + N - 1) / N - 1);
}

// Pool row of token `tok` of `seat` (bounds-checked page id) and how many rows remain in its page.
__device__ __forceinline__ long long pool_row_index(const DecodeArgs& a, int seat, int tok, int& n_in_page) {
  const int pidx = tok / a.page_size;
  const int off = tok - pidx * a.page_size;
  int pg = a.block_table[static_cast<long long>(seat) * a.bt_stride + pidx];
  if (pg < 0 || pg >= a.num_pages) {
    atomicOr(a.status, kStatusBadPage);
    pg = 0;
  }
  n_in_page = a.page_size - off;
  return static_cast<long long>(pg) * a.page_size + off;
}

// Issue the bulk copies of global chunk i (seat given by cur) into stage buffers ks/vs; completion on `bar`.
template <int ROWS>
__device__ __forceinline__ void issue_chunk(const DecodeArgs& a, const SeatCursor& cur, long long i, uint8_t* ks,
                                            uint8_t* vs, uint64_t* bar) {
  const int tok0 = static_cast<int>(i - cur.first) * ROWS;
  const int rows = min(ROWS, cur.len - tok0);
  const bool has_new = a.k_new != nullptr && (tok0 + rows == cur.len);
  const int pool_rows = has_new ? rows - 1 : rows;
  mbar_arrive_expect_tx(bar, static_cast<uint32_t>(2 * rows * kRowBytes));
  for (int t = tok0; t < tok0 + pool_rows;) {
    int room;
    const long long row = pool_row_index(a, cur.seat, t, room);
    const int n = min(room, tok0 + pool_rows - t);
    bulk_g2s(ks + (t - tok0) * kRowBytes, a.k_pool + row * (kRowBytes / 2), n * kRowBytes, bar);
    bulk_g2s(vs + (t - tok0) * kRowBytes, a.v_pool + row * (kRowBytes / 2), n * kRowBytes, bar);
    t += n;
  }
  if (has_new) {
    const long long off = static_cast<long long>(cur.seat) * a.kv_new_stride;
    bulk_g2s(ks + (rows - 1) * kRowBytes, a.k_new + off, kRowBytes, bar);
    bulk_g2s(vs + (rows - 1) * kRowBytes, a.v_new + off, kRowBytes, bar);
  }
}

// Registers per thread for MIN_CTAS resident 8-warp CTAs: each of the SM's 4 sub-partitions holds 16K registers for
// ceil(warps / 4) warps.
template <int MIN_CTAS>
constexpr int decode_max_regs() {
  constexpr int warps_per_subpartition = (MIN_CTAS * kDecodeWarps + 3) / 4;
  constexpr int r = (16384 / (warps_per_subpartition * 32)) / 8 * 8;
  return r > 255 ? 255 : r;
}

template <int ROWS, int NSTAGES, int MIN_CTAS>
__global__ void __maxnreg__(decode_max_regs<MIN_CTAS>()) paged_decode_kernel(const DecodeArgs a) {
  using SL = DecodeSmemLayout<ROWS, NSTAGES>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL::kBarOff);
  unsigned* done = reinterpret_cast<unsigned*>(smem + SL::kDoneOff);
  float* pbuf_all = reinterpret_cast<float*>(smem + SL::kPOff);
  volatile int* abort_flag = reinterpret_cast<int*>(smem + SL::kMiscOff);
  __shared__ long long warp_sums[kDecodeWarps];
  __shared__ long long plan_first;
  __shared__ int plan_seat;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;   // G: launched CTAs (the split is re-derived below from N)
  const bool append = a.k_new != nullptr;

  if (tid == 0) {
    for (int s = 0; s < NSTAGES; ++s) {
      mbar_init(&full[s], 1);
      done[s] = 0;
    }
    *abort_flag = 0;
    fence_mbar_init();
  }

  // ---- plan: total chunk count N, then the seat holding this CTA's first chunk.
  long long local = 0;
  for (int s = tid; s < a.B; s += kDecodeThreads) {
    const int L = seat_tokens(a, s);
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
  if (lane == 0) warp_sums[warp] = local;
  __syncthreads();
  long long N = 0;
#pragma unroll
  for (int w = 0; w < kDecodeWarps; ++w) N += warp_sums[w];
  // Effective CTA count: never more CTAs than chunks, so every CTA in [0, Ge) owns at least one chunk and the CTAs
  // between a seat's first and last owner all contribute a partial (the merge counts them).
  const int Ge = static_cast<int>(N < G ? N : G);
  if (c >= Ge) return;    // uniform across the CTA; nothing has been issued
  const long long c0 = (N * c) / Ge, c1 = (N * (c + 1)) / Ge;

  {
    long long base = 0;
    for (int t0 = 0; t0 < a.B; t0 += kDecodeThreads) {
      const int s = t0 + tid;
      const int n = s < a.B ? (seat_tokens(a, s) + ROWS - 1) / ROWS : 0;
      long long incl = n;   // block inclusive scan of n
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
      for (int w = 0; w < kDecodeWarps; ++w) {
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
  cur.len = seat_tokens(a, cur.seat);
  cur.nch = (cur.len + ROWS - 1) / ROWS;

  // ---- prologue: warp 0 issues the first NSTAGES chunks. Every warp keeps a look-ahead cursor on chunk i + NSTAGES
  //      because whichever warp finishes a stage last refills it.
  SeatCursor look = cur;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < NSTAGES && c0 + s < c1; ++s) {
      advance<ROWS>(a, look, c0 + s);
      issue_chunk<ROWS>(a, look, c0 + s, smem + SL::kKOff + s * SL::kStageBytes, smem + SL::kVOff + s * SL::kStageBytes,
                        &full[s]);
    }
  }
  look = cur;

  // ================= warp h = KV head h, q heads 2h and 2h+1
  // Scores: the LPR lanes of a row split its 128 dims (DPL each, P pieces of 16 bytes); lane l scores row l / LPR.
  // Within a quarter-warp the lanes read different rows at the same offset, which would hit one bank group, so each
  // lane walks its pieces in a rotated order (rot) that puts the 8 lanes of a quarter-warp on 8 distinct 16-byte
  // bank groups; q is loaded into registers in the same rotated order, so register indexing stays static.
  // P.V: lane l owns dims 4l..4l+3 of both q heads and walks the chunk's rows (consecutive lanes, consecutive bytes).
  const int h = warp;
  float* pbuf = pbuf_all + warp * 2 * ROWS;     // [row][q head] probabilities of the current chunk
  constexpr int LPR = 32 / ROWS;                // lanes per row: 4 (ROWS 8) or 2 (ROWS 16)
  constexpr int DPL = kHeadDim / LPR;           // dims per lane: 32 or 64
  constexpr int P = DPL / 8;                    // 16-byte pieces per lane: 4 or 8
  static_assert(ROWS == 8 || ROWS == 16, "chunk rows must be 8 or 16");
  const int my_row = lane / LPR;
  const int my_part = lane % LPR;
  const int rot = (ROWS == 8) ? ((lane >> 1) & 3) : (lane & 7);
  const int my_g = lane & 1;                    // q head whose score this lane holds after the pair reduction
  const bool my_owner = (ROWS == 16) || ((lane & 2) == 0);   // one lane per (row, head) feeds the running sum

  int it = 0;
  long long i = c0;
  bool aborted = false;
  while (i < c1 && !aborted) {
    advance<ROWS>(a, cur, i);
    // ---- a seat's chunks within this CTA: load its q (rotated, pre-scaled), reset the running state
    float2 qv[2][P][4];                         // [head][piece (rotated)][pair] pre-scaled by scale*log2(e)
    {
      const __nv_bfloat16* qb = a.q + static_cast<long long>(cur.seat) * a.q_stride + (2 * h) * kHeadDim + my_part * DPL;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
#pragma unroll
        for (int pc = 0; pc < P; ++pc) {
          const uint4 w = __ldg(reinterpret_cast<const uint4*>(qb + g * kHeadDim + ((pc + rot) % P) * 8));
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = bf16x2_to_float2(word_of(w, e));
            qv[g][pc][e] = make_float2(f.x * a.scale_log2, f.y * a.scale_log2);
          }
        }
      }
    }
    float4 o0 = make_float4(0, 0, 0, 0), o1 = o0;
    float m0 = -INFINITY, m1 = -INFINITY, lsum = 0.f;
    const long long seat_end = (cur.first + cur.nch < c1) ? cur.first + cur.nch : c1;

    for (; i < seat_end; ++i, ++it) {
      const int stage = it % NSTAGES;
      if (!mbar_wait_bounded(&full[stage], (it / NSTAGES) & 1)) {
        atomicOr(a.status, kStatusWaitTimeout);
        *abort_flag = 1;
        aborted = true;
        break;
      }
      const int tok0 = static_cast<int>(i - cur.first) * ROWS;
      const int rows = min(ROWS, cur.len - tok0);
      uint8_t* kst = smem + SL::kKOff + stage * SL::kStageBytes;
      uint8_t* vst = smem + SL::kVOff + stage * SL::kStageBytes;

      // ---- scores (rows >= `rows` hold stale bytes; their scores are discarded below)
      const uint8_t* krow = kst + my_row * kRowBytes + h * kHeadBytes + my_part * DPL * 2;
      float2 acc0 = make_float2(0.f, 0.f), acc1 = acc0;
#pragma unroll
      for (int pc = 0; pc < P; ++pc) {
        const uint4 w = *reinterpret_cast<const uint4*>(krow + ((pc + rot) % P) * 16);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 k = bf16x2_to_float2(word_of(w, e));
          acc0 = __ffma2_rn(qv[0][pc][e], k, acc0);
          acc1 = __ffma2_rn(qv[1][pc][e], k, acc1);
        }
      }
      float s0 = acc0.x + acc0.y, s1 = acc1.x + acc1.y;
      {   // pair reduction: after xor 1 each lane keeps head (lane & 1); further xors finish the row's LPR lanes
        const bool up = (lane & 1) != 0;
        const float send = up ? s0 : s1;
        s0 = (up ? s1 : s0) + __shfl_xor_sync(0xffffffffu, send, 1);
#pragma unroll
        for (int o = 2; o < LPR; o <<= 1) s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      }
      const bool valid = my_row < rows;
      const float x = valid ? s0 : -INFINITY;
      float cm = x;
#pragma unroll
      for (int o = LPR; o < 32; o <<= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
      const float cm_other = __shfl_xor_sync(0xffffffffu, cm, 1);
      const float cm0 = my_g ? cm_other : cm, cm1 = my_g ? cm : cm_other;
      const float mn0 = fmaxf(m0, cm0), mn1 = fmaxf(m1, cm1);
      const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      const float p = valid ? exp2f(x - (my_g ? mn1 : mn0)) : 0.f;
      lsum = lsum * (my_g ? a1 : a0) + (my_owner ? p : 0.f);
      if (my_owner && valid) pbuf[my_row * 2 + my_g] = p;
      __syncwarp();

      // ---- P.V
      {
        const uint8_t* vb = vst + h * kHeadBytes + lane * 8;
        float2 oa = make_float2(o0.x * a0, o0.y * a0), ob = make_float2(o0.z * a0, o0.w * a0);
        float2 oc = make_float2(o1.x * a1, o1.y * a1), od = make_float2(o1.z * a1, o1.w * a1);
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          if (r < rows) {
            const float2 pp = *reinterpret_cast<const float2*>(pbuf + 2 * r);
            const uint2 w = *reinterpret_cast<const uint2*>(vb + r * kRowBytes);
            const float2 v01 = bf16x2_to_float2(w.x), v23 = bf16x2_to_float2(w.y);
            const float2 p0 = make_float2(pp.x, pp.x), p1 = make_float2(pp.y, pp.y);
            oa = __ffma2_rn(v01, p0, oa);
            ob = __ffma2_rn(v23, p0, ob);
            oc = __ffma2_rn(v01, p1, oc);
            od = __ffma2_rn(v23, p1, od);
          }
        }
        o0 = make_float4(oa.x, oa.y, ob.x, ob.y);
        o1 = make_float4(oc.x, oc.y, od.x, od.y);
      }

      // ---- fused append: this chunk holds the new token; write head h of its row into the pools
      if (append && tok0 + rows == cur.len) {
        int room;
        const long long row = pool_row_index(a, cur.seat, cur.len - 1, room);
        const int off = h * kHeadDim + 4 * lane;
        *reinterpret_cast<uint2*>(a.k_pool + row * (kRowBytes / 2) + off) =
            *reinterpret_cast<const uint2*>(kst + (rows - 1) * kRowBytes + off * 2);
        *reinterpret_cast<uint2*>(a.v_pool + row * (kRowBytes / 2) + off) =
            *reinterpret_cast<const uint2*>(vst + (rows - 1) * kRowBytes + off * 2);
      }

      // ---- release the stage; the last of the 8 warps refills it with chunk i + NSTAGES
      __syncwarp();
      if (i + NSTAGES < c1) advance<ROWS>(a, look, i + NSTAGES);
      if (lane == 0) {
        __threadfence_block();
        const unsigned prev = atomicAdd(&done[stage], 1u);
        if ((prev % kDecodeWarps) == kDecodeWarps - 1 && i + NSTAGES < c1) {
          fence_proxy_async_smem();
          issue_chunk<ROWS>(a, look, i + NSTAGES, kst, vst, &full[stage]);
        }
      }
      if (*abort_flag) {
        aborted = true;
        break;
      }
    }   // chunks of this seat
    if (aborted) break;

    // ---- end of the seat's chunks in this CTA (q registers are dead here)
    float lg = lsum;                                   // lanes of equal parity hold the same q head
#pragma unroll
    for (int o = 2; o < 32; o <<= 1) lg += __shfl_xor_sync(0xffffffffu, lg, o);
    const float lo = __shfl_xor_sync(0xffffffffu, lg, 1);
    const float l0 = my_g ? lo : lg, l1 = my_g ? lg : lo;
    const int c_first = cta_of_chunk(cur.first, N, Ge);
    const int c_last = cta_of_chunk(cur.first + cur.nch - 1, N, Ge);
    __nv_bfloat16* op = a.out + static_cast<long long>(cur.seat) * a.out_stride + (2 * h) * kHeadDim + 4 * lane;
    if (c_first == c_last) {
      const float r0 = 1.f / l0, r1 = 1.f / l1;
      *reinterpret_cast<uint2*>(op) = float4_to_bf16x4(make_float4(o0.x * r0, o0.y * r0, o0.z * r0, o0.w * r0));
      *reinterpret_cast<uint2*>(op + kHeadDim) = float4_to_bf16x4(make_float4(o1.x * r1, o1.y * r1, o1.z * r1, o1.w * r1));
      continue;
    }
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
    if (ticket != static_cast<unsigned>(c_last - c_first)) continue;
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
    *reinterpret_cast<uint2*>(op + kHeadDim) = float4_to_bf16x4(make_float4(O1.x * r1, O1.y * r1, O1.z * r1, O1.w * r1));
    if (lane == 0) a.counters[static_cast<long long>(cur.seat) * kKvHeads + h] = 0u;   // ready for the next launch
  }

  // A warp that gave up may leave copies in flight into this CTA's shared memory: wait (bounded) for every issued
  // stage to land before the CTA exits.
  if (aborted && lane == 0) {
    for (int k = 0; k < NSTAGES; ++k)
      mbar_wait_bounded(&full[(it + k) % NSTAGES], ((it + k) / NSTAGES) & 1, 100000000ull);
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

template <int ROWS, int NSTAGES, int MIN_CTAS>
static int occupancy_of() {
  using SL = DecodeSmemLayout<ROWS, NSTAGES>;
  auto kern = paged_decode_kernel<ROWS, NSTAGES, MIN_CTAS>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SL::kBytes) != cudaSuccess) return -1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kDecodeThreads, SL::kBytes) != cudaSuccess) return -1;
  return n;
}

// Variants: 0 = 8-token chunks x 3 stages (96 KB, two CTAs per SM, default); 1 = 16-token chunks x 3 stages (192 KB,
// one CTA per SM); 2 = 8-token chunks x 2 stages (64 KB, two CTAs per SM).
int decode_occupancy(int variant) {
  switch (variant) {
    case 1: return occupancy_of<16, 3, 1>();
    case 2: return occupancy_of<8, 2, 2>();
    default: return occupancy_of<8, 3, 2>();
  }
}

int decode_rows_per_chunk(int variant) { return variant == 1 ? 16 : 8; }

int decode_ctas_per_sm(int variant) { return variant == 1 ? 1 : 2; }

cudaError_t launch_paged_decode(const DecodeArgs& a, int grid, int variant, cudaStream_t stream) {
  switch (variant) {
    case 1: return launch_decode<16, 3, 1>(a, grid, stream);
    case 2: return launch_decode<8, 2, 2>(a, grid, stream);
    default: return launch_decode<8, 3, 2>(a, grid, stream);
  }
}

}  // namespace q3
