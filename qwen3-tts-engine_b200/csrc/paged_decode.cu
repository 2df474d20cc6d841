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
// A chunk stream is read by 8 consumer warps, one per KV head: K and V of a chunk (ROWS token rows of 2 KB, all 8
// heads) are brought into a ring of NSTAGES shared-memory stages by one-dimensional TMA bulk copies (cp.async.bulk)
// whose completion is counted on an mbarrier per stage. Two ways to refill the stages:
//   * paged_decode_kernel (variants 0-2): 8-warp CTAs, no dedicated producer. Warp 0 issues the first NSTAGES chunks;
//     after that, the warp that is LAST to finish reading a stage (a shared-memory ticket per stage) refills it with
//     the chunk NSTAGES further on. Keeping the CTA at 8 warps lets two CTAs share an SM at 128 registers per thread
//     (the register file is split over the SM's four sub-partitions, 16K registers each).
//   * paged_decode_ws_kernel (variant 5, the default): one CTA per SM with two streams, each refilled by a producer
//     warp of its own (described where it is defined).
// Both run the same consumer code (decode_consume).
//
// Scores: lane l of warp h scores row l / LPR of the chunk over DPL of the 128 dims, for both q heads of the group,
// with packed fp32 FMAs (FFMA2); LPR lanes per row combine with shuffles. Online softmax in the exp2 domain.
// P.V: lane l owns dims 4l..4l+3 of both q heads.
//
// Fused append (k/v given): the new token goes at position cache_seqlens[b]; its row is copied from k_new/v_new into
// the stage, and each warp writes its head's 256 bytes of that row into the page pool. Only the CTA that owns the
// chunk holding the new token reads that row in this launch, so no other CTA can race with the write.
#include "decode_common.cuh"

namespace q3 {

template <int ROWS, int NSTAGES, bool FUSE = false>
struct DecodeSmemLayout {
  static constexpr int kStageBytes = ROWS * kRowBytes;                  // K (or V) of one chunk
  static constexpr int kKOff = 0;
  static constexpr int kVOff = NSTAGES * kStageBytes;
  static constexpr int kBarOff = 2 * NSTAGES * kStageBytes;             // full[NSTAGES] mbarriers
  static constexpr int kDoneOff = kBarOff + NSTAGES * 8;                // done[NSTAGES] reader tickets
  static constexpr int kPOff = kDoneOff + ((NSTAGES * 4 + 15) / 16) * 16;   // per-warp probabilities [ROWS][2]
  static constexpr int kMiscOff = kPOff + kDecodeWarps * 2 * ROWS * 4;
  // FUSE: per-warp normalised q [2][128] bf16, read back with 16-byte loads, so 16-byte (here 128-byte) aligned
  static constexpr int kQOff = ((kMiscOff + 64 + 127) / 128) * 128;
  static constexpr int kBytes = kQOff + (FUSE ? kDecodeWarps * 2 * kHeadBytes : 0);
  static_assert(kQOff % 16 == 0 && kKOff % 16 == 0 && kVOff % 16 == 0 && kStageBytes % 16 == 0,
                "16-byte shared-memory accesses need 16-byte aligned regions");
};

// The consumer side of one chunk stream for KV head h (one warp): every seat of the plan's chunk range, chunks taken
// from a ring of NSTAGES shared-memory stages (K stages at k_stages, V stages at v_stages) that `ring` fills and
// frees. c is the split slot whose partials this stream leaves. `it` counts the chunks waited for; `aborted` is set
// when a wait gave up (the caller then waits for the copies still in flight).
//
// Scores: lane l of warp h scores row l / LPR of the chunk over DPL of the 128 dims, for both q heads of the group;
// the LPR lanes of a row combine with shuffles. Within a quarter-warp the lanes read different rows at the same
// offset, which would hit one bank group, so each lane walks its pieces in a rotated order (rot) that puts the 8 lanes
// of a quarter-warp on 8 distinct 16-byte bank groups; q is loaded into registers in the same rotated order, so
// register indexing stays static. P.V: lane l owns dims 4l..4l+3 of both q heads and walks the chunk's rows
// (consecutive lanes, consecutive bytes).
template <int ROWS, int NSTAGES, bool FUSE, class Ring>
__device__ __forceinline__ void decode_consume(const DecodeArgs& a, const DecodePlan& plan, int c, int h, int lane,
                                               uint8_t* k_stages, uint8_t* v_stages, float* pbuf, uint8_t* q_slot,
                                               Ring& ring, int& it, bool& aborted) {
  constexpr int kStageBytes = ROWS * kRowBytes;
  const bool append = a.k_new != nullptr;
  const long long c1 = plan.c1;
  SeatCursor cur = plan.cur;
  constexpr int LPR = 32 / ROWS;                // lanes per row: 4 (ROWS 8) or 2 (ROWS 16)
  constexpr int DPL = kHeadDim / LPR;           // dims per lane: 32 or 64
  constexpr int P = DPL / 8;                    // 16-byte pieces per lane: 4 or 8
  static_assert(ROWS == 8 || ROWS == 16, "chunk rows must be 8 or 16");
  const int my_row = lane / LPR;
  const int my_part = lane % LPR;
  const int rot = (ROWS == 8) ? ((lane >> 1) & 3) : (lane & 7);
  const int my_g = lane & 1;                    // q head whose score this lane holds after the pair reduction
  const bool my_owner = (ROWS == 16) || ((lane & 2) == 0);   // one lane per (row, head) feeds the running sum

  it = 0;
  aborted = false;
  long long i = plan.c0;
  while (i < c1 && !aborted) {
    advance<ROWS>(a, cur, i);
    // ---- a seat's chunks within this stream: load its q (rotated, pre-scaled), reset the running state
    float2 qv[2][P][4];                         // [head][piece (rotated)][pair] pre-scaled by scale*log2(e)
    {
      const __nv_bfloat16* qrow = a.q + static_cast<long long>(cur.seat) * a.q_stride + (2 * h) * kHeadDim;
      if constexpr (FUSE) {
        // raw projection -> RMSNorm + RoPE of both q heads (4 dims per lane), staged in this warp's shared slot
        const long long ro = static_cast<long long>(cur.seat) * a.rope_stride;
        uint2* qs = reinterpret_cast<uint2*>(q_slot);
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const float4 x = bf16x4_to_float4(*reinterpret_cast<const uint2*>(qrow + g * kHeadDim + 4 * lane));
          qs[g * 32 + lane] =
              float4_to_bf16x4(rms_rope_head(x, a.qn_w, a.rope_cos + ro, a.rope_sin + ro, a.eps, lane));
        }
        __syncwarp();
        qrow = reinterpret_cast<const __nv_bfloat16*>(qs);
      }
      const __nv_bfloat16* qb = qrow + my_part * DPL;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
#pragma unroll
        for (int pc = 0; pc < P; ++pc) {
          const uint4* src = reinterpret_cast<const uint4*>(qb + g * kHeadDim + ((pc + rot) % P) * 8);
          const uint4 w = FUSE ? *src : __ldg(src);
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

    // scores of one chunk from its K stage: after the pair reduction lane l holds q head (l & 1), row l / LPR
    auto score = [&](const uint8_t* kst) -> float {
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
      const bool up = (lane & 1) != 0;
      const float send = up ? s0 : s1;
      s0 = (up ? s1 : s0) + __shfl_xor_sync(0xffffffffu, send, 1);
#pragma unroll
      for (int o = 2; o < LPR; o <<= 1) s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      return s0;
    };
    // online-softmax step for a chunk's scores: running maxima/sums, probabilities to pbuf; returns the factors by
    // which the outputs accumulated so far must be scaled
    auto softmax = [&](float sc, int rows, float& a0, float& a1) {
      const bool valid = my_row < rows;
      const float x = valid ? sc : -INFINITY;
      float cm = x;
#pragma unroll
      for (int o = LPR; o < 32; o <<= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
      const float cm_other = __shfl_xor_sync(0xffffffffu, cm, 1);
      const float cm0 = my_g ? cm_other : cm, cm1 = my_g ? cm : cm_other;
      const float mn0 = fmaxf(m0, cm0), mn1 = fmaxf(m1, cm1);
      a0 = exp2f(m0 - mn0);
      a1 = exp2f(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      const float p = valid ? exp2f(x - (my_g ? mn1 : mn0)) : 0.f;
      lsum = lsum * (my_g ? a1 : a0) + (my_owner ? p : 0.f);
      if (my_owner && valid) pbuf[my_row * 2 + my_g] = p;
    };
    // P.V of a chunk from its V stage (probabilities already in pbuf), accumulated into o0/o1
    auto pv = [&](const uint8_t* vst, int rows) {
      const uint8_t* vb = vst + h * kHeadBytes + lane * 8;
      float2 oa = make_float2(o0.x, o0.y), ob = make_float2(o0.z, o0.w);
      float2 oc = make_float2(o1.x, o1.y), od = make_float2(o1.z, o1.w);
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
    };
    auto scale_out = [&](float a0, float a1) {
      o0.x *= a0; o0.y *= a0; o0.z *= a0; o0.w *= a0;
      o1.x *= a1; o1.y *= a1; o1.z *= a1; o1.w *= a1;
    };
    // fused append: a chunk holding the new token writes head h of its row into the pools
    auto append_row = [&](const uint8_t* kst, const uint8_t* vst, int rows) {
      int room;
      const long long row = pool_row_index(a, cur.seat, cur.len - 1, room);
      const int off = h * kHeadDim + 4 * lane;
      *reinterpret_cast<uint2*>(a.k_pool + row * (kRowBytes / 2) + off) =
          *reinterpret_cast<const uint2*>(kst + (rows - 1) * kRowBytes + off * 2);
      *reinterpret_cast<uint2*>(a.v_pool + row * (kRowBytes / 2) + off) =
          *reinterpret_cast<const uint2*>(vst + (rows - 1) * kRowBytes + off * 2);
    };

    for (; i < seat_end; ++i, ++it) {
      const int stage = it % NSTAGES;
      if (!ring.wait(a, it)) {
        aborted = true;
        break;
      }
      const int tok0 = static_cast<int>(i - cur.first) * ROWS;
      const int rows = min(ROWS, cur.len - tok0);
      uint8_t* kst = k_stages + stage * kStageBytes;
      uint8_t* vst = v_stages + stage * kStageBytes;
      if constexpr (FUSE) {
        if (tok0 + rows == cur.len) {
          // the new token's raw k row (copied from the projection): RMSNorm + RoPE of head h in place, before it is
          // scored and appended; the generic-proxy write is fenced against the stage's next bulk refill
          uint2* kr = reinterpret_cast<uint2*>(kst + (rows - 1) * kRowBytes + h * kHeadBytes) + lane;
          const long long ro = static_cast<long long>(cur.seat) * a.rope_stride;
          *kr = float4_to_bf16x4(
              rms_rope_head(bf16x4_to_float4(*kr), a.kn_w, a.rope_cos + ro, a.rope_sin + ro, a.eps, lane));
          fence_proxy_async_smem();
          __syncwarp();
        }
      }
      float a0, a1;
      softmax(score(kst), rows, a0, a1);
      scale_out(a0, a1);
      __syncwarp();
      pv(vst, rows);
      if (append && tok0 + rows == cur.len) append_row(kst, vst, rows);
      ring.release(a, i, stage, kst, vst, lane);
      if (ring.aborted()) {
        aborted = true;
        break;
      }
    }
    if (aborted) break;

    // ---- end of the seat's chunks in this stream (q registers are dead here)
    float lg = lsum;                                   // lanes of equal parity hold the same q head
#pragma unroll
    for (int o = 2; o < 32; o <<= 1) lg += __shfl_xor_sync(0xffffffffu, lg, o);
    const float lo = __shfl_xor_sync(0xffffffffu, lg, 1);
    decode_finish_seat(a, plan, c, cur, h, lane, o0, o1, m0, m1, my_g ? lo : lg, my_g ? lg : lo);
  }
}

// Stages refilled by the consumers themselves: the warp that is last to finish reading a stage (a shared-memory
// ticket per stage) issues the chunk NSTAGES further on into it. Every warp keeps the look-ahead cursor.
template <int ROWS, int NSTAGES>
struct RefillRing {
  uint64_t* full;
  unsigned* done;
  volatile int* abort_flag;
  SeatCursor look;
  long long c1;
  __device__ __forceinline__ bool wait(const DecodeArgs& a, int it) {
    if (mbar_wait_bounded(&full[it % NSTAGES], (it / NSTAGES) & 1)) return true;
    atomicOr(a.status, kStatusWaitTimeout);
    *abort_flag = 1;
    return false;
  }
  __device__ __forceinline__ void release(const DecodeArgs& a, long long ci, int stage, uint8_t* kst, uint8_t* vst,
                                          int lane) {
    __syncwarp();
    if (ci + NSTAGES < c1) advance<ROWS>(a, look, ci + NSTAGES);
    if (lane == 0) {
      __threadfence_block();
      const unsigned prev = atomicAdd(&done[stage], 1u);
      if ((prev % kDecodeWarps) == kDecodeWarps - 1 && ci + NSTAGES < c1) {
        fence_proxy_async_smem();
        issue_chunk<ROWS>(a, look, ci + NSTAGES, kst, vst, &full[stage]);
      }
    }
  }
  __device__ __forceinline__ bool aborted() const { return *abort_flag != 0; }
};

template <int ROWS, int NSTAGES, int MIN_CTAS, bool FUSE = false>
__global__ void __maxnreg__(decode_max_regs<MIN_CTAS>()) paged_decode_kernel(const DecodeArgs a) {
  using SL = DecodeSmemLayout<ROWS, NSTAGES, FUSE>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL::kBarOff);
  unsigned* done = reinterpret_cast<unsigned*>(smem + SL::kDoneOff);
  float* pbuf_all = reinterpret_cast<float*>(smem + SL::kPOff);
  volatile int* abort_flag = reinterpret_cast<int*>(smem + SL::kMiscOff);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (tid == 0) {
    for (int s = 0; s < NSTAGES; ++s) {
      mbar_init(&full[s], 1);
      done[s] = 0;
    }
    *abort_flag = 0;
    fence_mbar_init();
  }

  DecodePlan plan;
  if (!decode_plan<ROWS>(a, plan)) return;
  const long long c0 = plan.c0, c1 = plan.c1;

  // ---- prologue: warp 0 issues the first NSTAGES chunks; after that, whichever warp finishes a stage last refills it
  if (warp == 0 && lane == 0) {
    SeatCursor look = plan.cur;
    for (int s = 0; s < NSTAGES && c0 + s < c1; ++s) {
      advance<ROWS>(a, look, c0 + s);
      issue_chunk<ROWS>(a, look, c0 + s, smem + SL::kKOff + s * SL::kStageBytes, smem + SL::kVOff + s * SL::kStageBytes,
                        &full[s]);
    }
  }
  RefillRing<ROWS, NSTAGES> ring{full, done, abort_flag, plan.cur, c1};

  // ---- warp h = KV head h, q heads 2h and 2h+1
  int it = 0;
  bool aborted = false;
  decode_consume<ROWS, NSTAGES, FUSE>(a, plan, static_cast<int>(blockIdx.x), warp, lane, smem + SL::kKOff,
                                      smem + SL::kVOff, pbuf_all + warp * 2 * ROWS,
                                      smem + SL::kQOff + warp * 2 * kHeadBytes, ring, it, aborted);

  // A warp that gave up may leave copies in flight into this CTA's shared memory: wait (bounded) for every issued
  // stage to land before the CTA exits.
  if (aborted && lane == 0) {
    for (int k = 0; k < NSTAGES; ++k)
      mbar_wait_bounded(&full[(it + k) % NSTAGES], ((it + k) / NSTAGES) & 1, 100000000ull);
  }
}

// ------------------------------------------------------------------ dedicated producers (variant 5)
// One CTA per SM runs two chunk streams: split slots 2x and 2x + 1 of a split over 2 x gridDim.x slots. Each stream
// has its own ring of NSTAGES stages and eight consumer warps (one per KV head, the math of decode_consume), and a
// producer warp that does nothing else. The producer waits until all eight consumers have released a stage (an
// `empty` mbarrier of count 8), then issues the chunk NSTAGES further on into it, so no consumer ever pays for a
// block-table load or a copy issue. 20 warps: warpgroup 0 holds the two producers (its warps 2-3 leave at once),
// warpgroups 1-2 are stream 0's consumers, 3-4 stream 1's. The CTA is launched at 96 registers per thread (640 threads
// fill the register file); warpgroup 0 gives registers back down to 32 (setmaxnreg.dec) and the consumers take 112
// (setmaxnreg.inc): 128 x 32 + 512 x 112 = 640 x 96, also per SM sub-partition (one producer-group warp and four
// consumer warps on each).
constexpr int kWsStreams = 2;
constexpr int kWsWarps = 4 + kWsStreams * kDecodeWarps;   // 20
constexpr int kWsThreads = kWsWarps * 32;                 // 640
constexpr int kWsLaunchRegs = 96, kWsProducerRegs = 32, kWsConsumerRegs = 112;
static_assert(128 * kWsProducerRegs + kWsStreams * kDecodeThreads * kWsConsumerRegs == kWsThreads * kWsLaunchRegs,
              "the register split must add up to what the CTA is launched with");

template <int ROWS, int NSTAGES, bool FUSE = false>
struct WsSmemLayout {
  static constexpr int kStageBytes = ROWS * kRowBytes;                // K (or V) of one chunk
  static constexpr int kStreamBytes = 2 * NSTAGES * kStageBytes;      // a stream's K stages, then its V stages
  static constexpr int kBarOff = kWsStreams * kStreamBytes;           // per stream: full[NSTAGES], empty[NSTAGES]
  static constexpr int kPOff = kBarOff + kWsStreams * 2 * NSTAGES * 8;
  static constexpr int kMiscOff = kPOff + kWsStreams * kDecodeWarps * 2 * ROWS * 4;
  // FUSE: per consumer warp the normalised q [2][128] bf16, read back with 16-byte loads
  static constexpr int kQOff = ((kMiscOff + 16 + 127) / 128) * 128;
  static constexpr int kBytes = kQOff + (FUSE ? kWsStreams * kDecodeWarps * 2 * kHeadBytes : 0);
};

// Stages filled by a producer warp: a consumer warp releases a stage by one arrival on its `empty` barrier.
template <int NSTAGES>
struct ProducerRing {
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort_flag;
  __device__ __forceinline__ bool wait(const DecodeArgs& a, int it) {
    if (mbar_wait_bounded(&full[it % NSTAGES], (it / NSTAGES) & 1)) return true;
    atomicOr(a.status, kStatusWaitTimeout);
    *abort_flag = 1;
    return false;
  }
  __device__ __forceinline__ void release(const DecodeArgs&, long long, int stage, uint8_t*, uint8_t*, int lane) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }
  __device__ __forceinline__ bool aborted() const { return *abort_flag != 0; }
};

// The producer of one stream (one thread): chunk k of the stream goes to stage k % NSTAGES once the consumers have
// released chunk k - NSTAGES from it (phase k / NSTAGES - 1 of that stage's empty barrier).
template <int ROWS, int NSTAGES>
__device__ __forceinline__ void decode_produce(const DecodeArgs& a, const DecodePlan& P, uint8_t* k_stages,
                                               uint8_t* v_stages, uint64_t* full, uint64_t* empty,
                                               volatile int* abort_flag) {
  constexpr int kStageBytes = ROWS * kRowBytes;
  SeatCursor look = P.cur;
  long long k = 0;
  bool ok = true;
  for (long long i = P.c0; i < P.c1; ++i, ++k) {
    const int stage = static_cast<int>(k % NSTAGES);
    if (k >= NSTAGES && !mbar_wait_bounded(&empty[stage], static_cast<uint32_t>((k / NSTAGES - 1) & 1))) {
      atomicOr(a.status, kStatusWaitTimeout);
      *abort_flag = 1;
    }
    if (*abort_flag) {
      ok = false;
      break;
    }
    advance<ROWS>(a, look, i);
    fence_proxy_async_smem();
    issue_chunk<ROWS>(a, look, i, k_stages + stage * kStageBytes, v_stages + stage * kStageBytes, &full[stage]);
  }
  if (!ok) {
    // the last NSTAGES chunks issued may still be landing in this CTA's shared memory: wait for them (bounded)
    for (long long j = k > NSTAGES ? k - NSTAGES : 0; j < k; ++j)
      mbar_wait_bounded(&full[j % NSTAGES], static_cast<uint32_t>((j / NSTAGES) & 1), 100000000ull);
  }
}

template <int ROWS, int NSTAGES, bool FUSE = false>
__global__ void __launch_bounds__(kWsThreads, 1) paged_decode_ws_kernel(const DecodeArgs a) {
  using SL = WsSmemLayout<ROWS, NSTAGES, FUSE>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SL::kBarOff);   // stream s: full at 2*NSTAGES*s, empty after
  volatile int* abort_flag = reinterpret_cast<int*>(smem + SL::kMiscOff);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (tid == 0) {
    for (int s = 0; s < kWsStreams; ++s) {
      for (int k = 0; k < NSTAGES; ++k) {
        mbar_init(&bars[2 * NSTAGES * s + k], 1);
        mbar_init(&bars[2 * NSTAGES * s + NSTAGES + k], kDecodeWarps);
      }
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  // the stream this warp works for: producers 0 and 1 feed streams 0 and 1, consumer warp 4 + 8s + h reads stream s
  const int mine = warp < 4 ? (warp < kWsStreams ? warp : 0) : (warp - 4) / kDecodeWarps;
  DecodePlan my;
  const unsigned active = decode_plan_streams<ROWS, kWsWarps, kWsStreams>(a, a.split_slots, mine, my);
  if (active == 0u) return;   // uniform across the CTA; the plan's barriers also published the barrier init

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kWsProducerRegs));
    if (warp < kWsStreams && lane == 0 && ((active >> warp) & 1u)) {
      uint8_t* base = smem + warp * SL::kStreamBytes;
      uint64_t* full = bars + 2 * NSTAGES * warp;
      decode_produce<ROWS, NSTAGES>(a, my, base, base + NSTAGES * SL::kStageBytes, full, full + NSTAGES, abort_flag);
    }
    return;
  }
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kWsConsumerRegs));
  const int s = mine, h = (warp - 4) % kDecodeWarps;
  if (!((active >> s) & 1u)) return;
  uint8_t* base = smem + s * SL::kStreamBytes;
  uint64_t* full = bars + 2 * NSTAGES * s;
  ProducerRing<NSTAGES> ring{full, full + NSTAGES, abort_flag};
  int it = 0;
  bool aborted = false;
  decode_consume<ROWS, NSTAGES, FUSE>(a, my, kWsStreams * static_cast<int>(blockIdx.x) + s, h, lane, base,
                                      base + NSTAGES * SL::kStageBytes,
                                      reinterpret_cast<float*>(smem + SL::kPOff) + (s * kDecodeWarps + h) * 2 * ROWS,
                                      smem + SL::kQOff + (s * kDecodeWarps + h) * 2 * kHeadBytes, ring, it, aborted);
  // a consumer that gave up leaves (bounded) only once the stages the producer may have issued have landed
  if (aborted && lane == 0) {
    for (int k = 0; k < NSTAGES; ++k)
      mbar_wait_bounded(&full[(it + k) % NSTAGES], ((it + k) / NSTAGES) & 1, 100000000ull);
  }
}

// ------------------------------------------------------------------ host-side launch
template <int ROWS, int NSTAGES, int MIN_CTAS, bool FUSE = false>
static cudaError_t launch_decode(const DecodeArgs& a, int grid, cudaStream_t stream) {
  using SL = DecodeSmemLayout<ROWS, NSTAGES, FUSE>;
  auto kern = paged_decode_kernel<ROWS, NSTAGES, MIN_CTAS, FUSE>;
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
int occupancy_of() {
  using SL = DecodeSmemLayout<ROWS, NSTAGES>;
  auto kern = paged_decode_kernel<ROWS, NSTAGES, MIN_CTAS>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SL::kBytes) != cudaSuccess) return -1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kDecodeThreads, SL::kBytes) != cudaSuccess) return -1;
  return n;
}

// Variant 5: grid = split slots, two per CTA. The register split assumes the CTA is launched at exactly
// kWsLaunchRegs per thread; any other count (a different compiler) refuses the launch instead of risking a
// setmaxnreg.inc that could never be satisfied.
template <int ROWS, int NSTAGES, bool FUSE = false>
static cudaError_t launch_decode_ws(const DecodeArgs& a, int slots, cudaStream_t stream) {
  using SL = WsSmemLayout<ROWS, NSTAGES, FUSE>;
  auto kern = paged_decode_ws_kernel<ROWS, NSTAGES, FUSE>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kWsLaunchRegs) return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SL::kBytes);
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  DecodeArgs b = a;
  b.split_slots = slots;
  kern<<<(slots + kWsStreams - 1) / kWsStreams, kWsThreads, SL::kBytes, stream>>>(b);
  return cudaGetLastError();
}

template <int ROWS, int NSTAGES>
int occupancy_ws() {
  using SL = WsSmemLayout<ROWS, NSTAGES>;
  auto kern = paged_decode_ws_kernel<ROWS, NSTAGES>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SL::kBytes) != cudaSuccess) return -1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kWsThreads, SL::kBytes) != cudaSuccess) return -1;
  return n;
}

template <int NSTAGES, int MIN_CTAS>
cudaError_t launch_decode_mma(const DecodeArgs& a, int grid, cudaStream_t stream);
template <int NSTAGES, int MIN_CTAS>
int occupancy_mma();

// Variants: 0 = 8-token chunks x 3 stages (96 KB, two CTAs per SM, default); 1 = 16-token chunks x 3 stages (192 KB,
// one CTA per SM); 2 = 8-token chunks x 2 stages (64 KB, two CTAs per SM); 3 / 4 = warp-MMA scoring with early stage
// release (paged_decode_mma.cu), 8-token chunks x 3 / 2 stages, two CTAs per SM; 5 = dedicated producers, one CTA
// per SM running two 8-token x 3-stage chunk streams (its grid argument counts chunk streams, two per CTA).
int decode_occupancy(int variant) {
  switch (variant) {
    case 5: return occupancy_ws<8, 3>();
    case 1: return occupancy_of<16, 3, 1>();
    case 2: return occupancy_of<8, 2, 2>();
    case 3: return occupancy_mma<3, 2>();
    case 4: return occupancy_mma<2, 2>();
    default: return occupancy_of<8, 3, 2>();
  }
}

int decode_rows_per_chunk(int variant) { return variant == 1 ? 16 : 8; }

int decode_ctas_per_sm(int variant) { return variant == 1 ? 1 : 2; }

cudaError_t launch_paged_decode_fused(const DecodeArgs& a, int grid, int variant, cudaStream_t stream) {
  if (variant == 5) return launch_decode_ws<8, 3, true>(a, grid, stream);
  return launch_decode<8, 3, 2, true>(a, grid, stream);
}

cudaError_t launch_paged_decode(const DecodeArgs& a, int grid, int variant, cudaStream_t stream) {
  switch (variant) {
    case 1: return launch_decode<16, 3, 1>(a, grid, stream);
    case 2: return launch_decode<8, 2, 2>(a, grid, stream);
    case 3: return launch_decode_mma<3, 2>(a, grid, stream);
    case 4: return launch_decode_mma<2, 2>(a, grid, stream);
    case 5: return launch_decode_ws<8, 3>(a, grid, stream);
    default: return launch_decode<8, 3, 2>(a, grid, stream);
  }
}

}  // namespace q3
