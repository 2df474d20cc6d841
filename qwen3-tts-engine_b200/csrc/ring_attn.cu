// Windowed ring attention of the streaming codec decoder, fp16, sm_100a.
//
// Replaces the attention of StreamCore.forward in ring mode (engine/decoder_stream.py:147-181) for one transformer
// layer: every stream keeps the rotated keys and values of its recent frames in a ring of RING slots (frame f in slot
// f % RING); a chunk of n new frames at absolute positions pos .. pos+n-1 attends over
//   * ring slot j, which holds frame qj = (pos-1) - ((pos-1-j) mod RING), when qj >= 0 and qj >= (pos+i) - PAST
//     (decoder_stream.py:152-155: the 72-frame window, a query sees itself + 71 past frames), and
//   * the chunk's own keys jj <= i (decoder_stream.py:156),
// with the arithmetic of the reference's fp16 matmuls (decoder_stream.py:173-175): each score is an fp16-rounded dot
// product, scaled and masked in fp32; P = softmax(.) rounded to fp16; o = fp16(fp16(P_ring V_ring) + fp16(P_new V_new)).
// With write_new set, the chunk's K/V columns are also stored into ring slots (pos + j) % RING (the index_copy_ of
// StreamDecoder._step, decoder_stream.py:330-333); those slots hold frames older than the window (n <= RING - PAST),
// so no query of this launch can see them, and each CTA writes only its own head after reading it.
//
// The ring rows that some query of the chunk sees form one contiguous range of distances d = 0 .. nvis-1 back from the
// newest frame (the union over the chunk is query 0's window); the kernels read them in that order (row d), followed
// by the chunk's rows (the TMA pipeline in slot order). Ring rows no query sees are never used. The kernels
// (launch_ring_attn picks one by chunk size and the q3_set_ring_frame_kernel / q3_set_ring_chunk_kernel selections;
// the defaults are the fastest measured):
//   * ring_attn_frame_stream_kernel (one frame, default): 4 (head_dim 64) or 8 (128) warps per (stream, head), every
//     row loaded straight into registers, nothing staged;
//   * ring_attn_frame_heads_kernel (one frame; windows past 79 rows under the default): one warp per head, G heads per CTA,
//     each staged row (the G heads of one slot) by one bulk copy into shared memory, scalar math;
//   * ring_attn_frame_mma_kernel (one frame) and ring_attn_chunk_mma_kernel (2..16 frames): the same staging into rows
//     padded by 16 bytes, both contractions on the tensor cores with P handed from the score fragments to the P.V
//     fragments in registers;
//   * ring_attn_frame_tma_kernel (one frame): a persistent pipeline staging (stream, head) items by 2-D tensor boxes;
// each described where it is defined; and, one CTA per (stream, head) with 4 warps (used also for every call another
// selection does not fit):
//   * ring_attn_mma_kernel (2..17 frames, default): rows staged by 16-byte asynchronous copies; the two ring contractions run
//     on the tensor cores (mma.sync m16n8k16, fp16 in, fp32 accumulation): S^T = K.Q^T over 16-key row tiles (the
//     chunk's keys included; queries as the 8-column operand) and O_ring^T = V_ring^T.P_ring^T over 16-key steps
//     (16 dims as the A operand by ldmatrix.x4.trans; V rows past nvis zeroed, so a zero probability never meets stale
//     data);
//     O_new = P_new.V_new (n <= 17 keys) is a few scalar FMAs per output. Rows of K, V and Q are 16-byte chunks
//     XOR-swizzled by (row & 7), which keeps every fragment load free of bank conflicts. About 25 KB of shared memory
//     at 88 slots, 4 frames, head_dim 64: eight CTAs per SM.
//   * ring_attn_frame_kernel (one frame): rows staged by one bulk copy each, scalar math.
#include "q3_common.cuh"
#include "q3_kernels.h"
#include "tensor_map.cuh"

#include <cuda_fp16.h>

#include <cstring>
#include <type_traits>

namespace q3 {

constexpr int kRingThreads = 128;

__device__ __forceinline__ float round_fp16(float x) { return __half2float(__float2half_rn(x)); }

// (pos - 1) mod RING, non-negative, for every int64 position, RING >= 2: division by the launch-invariant RING as a
// multiply-high by magic = ceil(2^(63 + l) / RING), l = ceil(log2 RING), and a shift by l - 1, exact for dividends up to
// 2^63 (Granlund and Montgomery, "Division by invariant integers using multiplication", 1994). pos - 1 >= 0 is divided
// as it is; below that, (pos - 1) mod RING = RING - 1 - ((-pos) mod RING).
__device__ __forceinline__ int ring_pm1_mod(long long pos, int ring, unsigned long long magic, int shift) {
  const unsigned long long up = static_cast<unsigned long long>(pos);
  const bool ge1 = pos >= 1;
  const unsigned long long z = ge1 ? up - 1ull : 0ull - up;  // pos - 1, or -pos: both in [0, 2^63]
  const unsigned long long q = __umul64hi(z, magic) >> shift;
  const int r = static_cast<int>(z - q * static_cast<unsigned long long>(ring));
  return ge1 ? r : ring - 1 - r;
}

// (pos - 1) mod RING for any ring size (the staged kernels; ring_magic / ring_shift are set for RING >= 2)
__device__ __forceinline__ int ring_pm1(long long pos, const RingArgs& a) {
  return a.ring == 1 ? 0 : ring_pm1_mod(pos, a.ring, a.ring_magic, a.ring_shift);
}

// Slot of frame pos + f given (pos - 1) mod RING (0 <= f <= the largest chunk)
__device__ __forceinline__ int ring_slot_after(int pm1_mod, int f, int ring) { return (pm1_mod + 1 + f) % ring; }


__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2_trans(const void* p, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(smem_addr(p)));
}

// Shared-memory geometry of one launch (every CTA uses the same layout): K, V: [KA][HD] halves (ring rows by distance
// 0 .. RP-1, then the chunk's rows RP .. RP+n-1, padded to 8), Q: [n][HD]; S: [n][KA] floats; P_ring: [n][RP + 8]
// halves; P_new: [n][n] floats.
struct RingGeom {
  int RP, KA, LPR;
  __host__ __device__ RingGeom(int ring, int past, int n) {
    const int nv = past < ring ? past : ring;   // ring rows any query can see
    RP = ((nv > 0 ? nv : 1) + 15) & ~15;
    KA = RP + ((n + 7) & ~7);
    LPR = RP + 8;
  }
  __host__ __device__ size_t bytes(int hd, int n) const {
    return (2ull * KA + n) * hd * sizeof(__half) + static_cast<size_t>(n) * KA * sizeof(float) +
           static_cast<size_t>(n) * LPR * sizeof(__half) + static_cast<size_t>(n) * n * sizeof(float);
  }
};

template <int HD>
__device__ __forceinline__ __half* swz(__half* base, int row, int chunk) {
  return base + (row * (HD / 8) + (chunk ^ (row & 7))) * 8;
}

template <int HD>
__global__ void __launch_bounds__(kRingThreads, HD == 64 ? 9 : 4) ring_attn_mma_kernel(const RingArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int CH = HD / 8;                                 // 16-byte chunks per row
  const int b = blockIdx.x, hh = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;                     // mma fragment coordinates
  const int n = a.n, RING = a.ring;
  const RingGeom G(RING, a.past, n);
  __half* sK = reinterpret_cast<__half*>(smem);
  __half* sV = sK + G.KA * HD;
  __half* sQ = sV + G.KA * HD;
  float* sS = reinterpret_cast<float*>(sQ + n * HD);
  __half* sPr = reinterpret_cast<__half*>(sS + n * G.KA);
  float* sPn = reinterpret_cast<float*>(sPr + n * G.LPR);

  const long long row = a.ring_rows[b];
  const long long pos = a.pos[b];
  // Distance d back from the newest frame (pos-1) lives in slot (pos-1-d) mod RING; query i sees it when
  // d <= min(pos-1, PAST-1-i) (decoder_stream.py:152-155), so rows d < nvis = min(pos, PAST, RING) cover every query.
  const int pm1_mod = ring_pm1(pos, a);
  int nvis = a.past < RING ? a.past : RING;
  if (pos < nvis) nvis = pos < 0 ? 0 : static_cast<int>(pos);

  const __half* kr = a.k_ring + row * a.ring_stream_stride + hh * HD;
  const __half* vr = a.v_ring + row * a.ring_stream_stride + hh * HD;
  for (int i = tid; i < G.RP * CH; i += kRingThreads) {
    const int d = i / CH, c = i - d * CH;
    if (d < nvis) {
      int j = pm1_mod - d;
      if (j < 0) j += RING;
      cp_async16(swz<HD>(sK, d, c), kr + j * a.ring_slot_stride + c * 8);
      cp_async16(swz<HD>(sV, d, c), vr + j * a.ring_slot_stride + c * 8);
    } else {
      *reinterpret_cast<uint4*>(swz<HD>(sV, d, c)) = make_uint4(0, 0, 0, 0);
    }
  }
  for (int i = tid; i < n * CH; i += kRingThreads) {
    const int f = i / CH, c = i - f * CH;
    const long long off = b * a.qkv_batch_stride + f * a.qkv_frame_stride + hh * HD + c * 8;
    cp_async16(swz<HD>(sK, G.RP + f, c), a.k_new + off);
    cp_async16(swz<HD>(sV, G.RP + f, c), a.v_new + off);
    cp_async16(swz<HD>(sQ, f, c), a.q + off);
  }
  cp_async_wait_all();
  __syncthreads();

  // ---- S^T = K.Q^T on the tensor cores, keys as the 16-row A operand (one ldmatrix.x4 per 16 dims from the swizzled K
  //      rows) and the chunk's queries as the 8-column B operand (loaded once per query tile): warp w takes key tiles
  //      w, w+4, ... Each score is an fp16-rounded dot product (the reference's fp16 matmul), scaled and masked in fp32.
  //      The last key tile may run up to 8 rows past KA (into V's first rows): those keys are never stored, and a
  //      non-finite value there stays in its own accumulator element.
  constexpr int NW = kRingThreads / 32;
  const int QT = (n + 7) / 8;                                // query tiles of 8
  const int KT = (G.KA + 15) / 16;                           // key tiles of 16
  for (int qt = 0; qt < QT; ++qt) {
    const int qi = qt * 8 + g;                               // the query whose B column this lane supplies
    uint32_t qf[HD / 16][2];
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      qf[ks][0] = qi < n ? *reinterpret_cast<const uint32_t*>(swz<HD>(sQ, qi, 2 * ks) + 2 * t) : 0u;
      qf[ks][1] = qi < n ? *reinterpret_cast<const uint32_t*>(swz<HD>(sQ, qi, 2 * ks + 1) + 2 * t) : 0u;
    }
    for (int kt = warp; kt < KT; kt += NW) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const int arow = kt * 16 + (lane & 15);                // lanes 0-15: dims 16ks..+7, lanes 16-31: 16ks+8..+15
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks) {
        uint32_t af[4];
        ldsm_x4(smem_addr(swz<HD>(sK, arow, 2 * ks + (lane >> 4))), af);
        mma_f16(acc, af[0], af[1], af[2], af[3], qf[ks][0], qf[ks][1]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = kt * 16 + g + (e >> 1) * 8;            // key (accumulator row)
        const int i = qt * 8 + 2 * t + (e & 1);              // query (accumulator column)
        if (i < n && c < G.KA) {
          const bool ok = c < G.RP ? (c < nvis && c <= a.past - 1 - i)   // ring row at distance c
                                   : (c - G.RP <= i);                    // the chunk's own keys, causally
          sS[i * G.KA + c] = ok ? round_fp16(acc[e]) * a.scale : -INFINITY;
        }
      }
    }
  }
  __syncthreads();

  // ---- softmax per query row (one warp per row), P rounded to fp16: the ring part as halves (MMA operand), the
  //      chunk part as floats
  for (int i = warp; i < n; i += NW) {
    float* srow = sS + i * G.KA;
    float m = -INFINITY;
    for (int c = lane; c < G.KA; c += 32) m = fmaxf(m, srow[c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
    for (int c = lane; c < G.KA; c += 32) {
      const float e = srow[c] == -INFINITY ? 0.f : expf(srow[c] - m);
      srow[c] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.f / sum;                             // the query always sees itself: sum > 0
    for (int c = lane; c < G.KA; c += 32) {
      const float p = round_fp16(srow[c] * inv);
      if (c < G.RP)
        sPr[i * G.LPR + c] = __float2half_rn(p);
      else if (c - G.RP < n)
        sPn[i * n + (c - G.RP)] = p;
    }
  }
  __syncthreads();

  // ---- O^T = V_ring^T.P_ring^T on the tensor cores: 16 dims as the A operand (ldmatrix.x4.trans of the V rows), the
  //      queries as the 8-column B operand (two 32-bit loads of P per 16 keys); warp w takes 16-dim tiles w, w+4, ...
  //      o = fp16(fp16(ring) + fp16(P_new.V_new)), the chunk's part a few scalar FMAs per output
  constexpr int DT16 = HD / 16 / NW;                         // 16-dim tiles per warp
  for (int qt = 0; qt < QT; ++qt) {
    const int qi = qt * 8 + g;                               // the query whose B column this lane supplies
    float acc[DT16][4];
#pragma unroll
    for (int u = 0; u < DT16; ++u) acc[u][0] = acc[u][1] = acc[u][2] = acc[u][3] = 0.f;
    const int lkey = (lane & 7) + ((lane >> 4) << 3), lch = (lane >> 3) & 1;   // this lane's ldmatrix row
    for (int ks = 0; ks < G.RP / 16; ++ks) {
      const __half* pr = sPr + qi * G.LPR + ks * 16 + 2 * t;
      const uint32_t b0 = qi < n ? *reinterpret_cast<const uint32_t*>(pr) : 0u;
      const uint32_t b1 = qi < n ? *reinterpret_cast<const uint32_t*>(pr + 8) : 0u;
#pragma unroll
      for (int u = 0; u < DT16; ++u) {
        uint32_t af[4];
        ldsm_x4_trans(smem_addr(swz<HD>(sV, ks * 16 + lkey, 2 * (warp + u * NW) + lch)), af);
        mma_f16(acc[u], af[0], af[1], af[2], af[3], b0, b1);
      }
    }
#pragma unroll
    for (int u = 0; u < DT16; ++u) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = 16 * (warp + u * NW) + g + (e >> 1) * 8;   // dim (accumulator row)
        const int i = qt * 8 + 2 * t + (e & 1);                  // query (accumulator column)
        if (i < n) {
          float ns = 0.f;                                        // the chunk's keys jj <= i
          for (int jj = 0; jj <= i; ++jj)
            ns = fmaf(sPn[i * n + jj], __half2float(swz<HD>(sV, G.RP + jj, d >> 3)[d & 7]), ns);
          a.out[b * a.out_batch_stride + i * a.out_frame_stride + hh * HD + d] =
              __float2half_rn(round_fp16(acc[u][e]) + round_fp16(ns));
        }
      }
    }
  }

  // ---- the chunk's columns into the ring (slots of frames outside every window of this launch, never staged)
  if (a.write_new) {
    __half* kw = a.k_ring + row * a.ring_stream_stride + hh * HD;
    __half* vw = a.v_ring + row * a.ring_stream_stride + hh * HD;
    for (int i = tid; i < n * CH; i += kRingThreads) {
      const int f = i / CH, c = i - f * CH;
      const int slot = ring_slot_after(pm1_mod, f, RING);
      reinterpret_cast<uint4*>(kw + slot * a.ring_slot_stride)[c] =
          *reinterpret_cast<const uint4*>(swz<HD>(sK, G.RP + f, c));
      reinterpret_cast<uint4*>(vw + slot * a.ring_slot_stride)[c] =
          *reinterpret_cast<const uint4*>(swz<HD>(sV, G.RP + f, c));
    }
  }
}

// One query frame (the streaming case, n = 1). The frame sees every staged ring row (distances d < nvis) and itself,
// so nothing is masked. Each row (K, V: one per distance, then the frame's own; q) arrives by its own 1-D bulk copy,
// all completing on one mbarrier: a few instructions per thread instead of an address computation per 16 bytes. For a
// single query row this scalar form finishes sooner than 16-row tensor-core tiles that are 15/16 padding. Thread r
// scores key r over 16-byte pieces in the rotated order (pc + r) % CH (the 8 lanes of a quarter-warp read 8 distinct
// bank groups), one warp runs the softmax, and P.V is split as (key group, 8-dim piece) per thread with the key groups
// summed by shuffles and a per-warp shared row.
template <int HD>
__global__ void __launch_bounds__(kRingThreads) ring_attn_frame_kernel(const RingArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int CH = HD / 8;                                 // 16-byte pieces per row
  constexpr int NW = kRingThreads / 32;
  constexpr uint32_t kRow = HD * sizeof(__half);
  const int b = blockIdx.x, hh = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int RING = a.ring;
  const int NV = a.past < RING ? a.past : RING;              // ring rows any frame can see (launch-wide)
  __half* sK = reinterpret_cast<__half*>(smem);              // [NV + 1][HD]: ring rows by distance, then the frame's
  __half* sV = sK + (NV + 1) * HD;
  __half* sQ = sV + (NV + 1) * HD;                           // [HD]
  float* sP = reinterpret_cast<float*>(sQ + HD);             // [NV + 1] scores, then probabilities
  float* sR = sP + ((NV + 1 + 3) & ~3);                      // [NW][HD] per-warp partial P_ring.V_ring
  uint64_t* bar = reinterpret_cast<uint64_t*>(sR + NW * HD);

  const long long row = a.ring_rows[b];
  const long long pos = a.pos[b];
  const int pm1_mod = ring_pm1(pos, a);
  int nvis = NV;                                             // distance d lives in slot (pos-1-d) mod RING
  if (pos < nvis) nvis = pos < 0 ? 0 : static_cast<int>(pos);
  const int nk = nvis + 1;                                   // keys: nvis ring rows, then the frame itself

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(2 * nk + 1) * kRow);
  }
  __syncthreads();
  const long long fo = b * a.qkv_batch_stride + hh * HD;     // the frame's q / k / v rows
  const __half* kr = a.k_ring + row * a.ring_stream_stride + hh * HD;
  const __half* vr = a.v_ring + row * a.ring_stream_stride + hh * HD;
  for (int i = tid; i < 2 * nk + 1; i += kRingThreads) {
    const __half* src;
    __half* dst;
    if (i == 2 * nk) {
      src = a.q + fo;
      dst = sQ;
    } else {
      const int r = i >> 1;
      const bool v = (i & 1) != 0;
      if (r < nvis) {
        int j = pm1_mod - r;
        if (j < 0) j += RING;
        src = (v ? vr : kr) + j * a.ring_slot_stride;
      } else {
        src = (v ? a.v_new : a.k_new) + fo;
      }
      dst = (v ? sV : sK) + r * HD;
    }
    bulk_g2s(dst, src, kRow, bar);
  }
  if (!__syncthreads_and(mbar_wait_bounded(bar, 0))) {       // uniform: every thread leaves together
    if (tid == 0) {
      atomicOr(a.status, kStatusWaitTimeout);
      mbar_wait_bounded(bar, 0, 100000000ull);                // the copies in flight land before the CTA exits
    }
    return;
  }

  // ---- scores: fp16-rounded dot products (the reference's fp16 matmul), scaled in fp32
  for (int r = tid; r < nk; r += kRingThreads) {
    const __half* krow = sK + r * HD;
    float2 acc0 = make_float2(0.f, 0.f), acc1 = acc0;
#pragma unroll
    for (int pc = 0; pc < CH; ++pc) {
      const int pp = (pc + r) & (CH - 1);
      const uint4 kw = *reinterpret_cast<const uint4*>(krow + pp * 8);
      const uint4 qw = *reinterpret_cast<const uint4*>(sQ + pp * 8);
      const __half2* kh = reinterpret_cast<const __half2*>(&kw);
      const __half2* qh = reinterpret_cast<const __half2*>(&qw);
      acc0 = __ffma2_rn(__half22float2(kh[0]), __half22float2(qh[0]), acc0);
      acc1 = __ffma2_rn(__half22float2(kh[1]), __half22float2(qh[1]), acc1);
      acc0 = __ffma2_rn(__half22float2(kh[2]), __half22float2(qh[2]), acc0);
      acc1 = __ffma2_rn(__half22float2(kh[3]), __half22float2(qh[3]), acc1);
    }
    sP[r] = round_fp16((acc0.x + acc0.y) + (acc1.x + acc1.y)) * a.scale;
  }
  __syncthreads();

  // ---- softmax (one warp), P rounded to fp16
  if (warp == 0) {
    float m = -INFINITY;
    for (int r = lane; r < nk; r += 32) m = fmaxf(m, sP[r]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
    for (int r = lane; r < nk; r += 32) {
      const float e = expf(sP[r] - m);
      sP[r] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.f / sum;
    for (int r = lane; r < nk; r += 32) sP[r] = round_fp16(sP[r] * inv);
  }
  __syncthreads();

  // ---- P_ring.V_ring: thread = (key group kg, 8-dim piece p); groups summed within the warp, then across warps
  constexpr int G = kRingThreads / CH;                       // key groups
  const int p = tid % CH, kg = tid / CH;
  float2 o[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  for (int r = kg; r < nvis; r += G) {
    const float pr = sP[r];
    const float2 pp2 = make_float2(pr, pr);
    const uint4 vw = *reinterpret_cast<const uint4*>(sV + r * HD + p * 8);
    const __half2* vh = reinterpret_cast<const __half2*>(&vw);
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = __ffma2_rn(__half22float2(vh[e]), pp2, o[e]);
  }
#pragma unroll
  for (int off = CH; off < 32; off <<= 1)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      o[e].x += __shfl_xor_sync(0xffffffffu, o[e].x, off);
      o[e].y += __shfl_xor_sync(0xffffffffu, o[e].y, off);
    }
  if (lane < CH) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sR[warp * HD + p * 8 + 2 * e] = o[e].x;
      sR[warp * HD + p * 8 + 2 * e + 1] = o[e].y;
    }
  }
  __syncthreads();
  // ---- o = fp16(fp16(P_ring.V_ring) + fp16(P_self.V_self))
  const float pself = sP[nvis];
  for (int d = tid; d < HD; d += kRingThreads) {
    float ring = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) ring += sR[w * HD + d];
    const float self = pself * __half2float(sV[nvis * HD + d]);
    a.out[b * a.out_batch_stride + hh * HD + d] = __float2half_rn(round_fp16(ring) + round_fp16(self));
  }

  // ---- the frame's columns into the ring (a slot outside every window of this launch, never staged)
  if (a.write_new) {
    const int slot = ring_slot_after(pm1_mod, 0, RING);
    __half* kw = a.k_ring + row * a.ring_stream_stride + hh * HD + slot * a.ring_slot_stride;
    __half* vw = a.v_ring + row * a.ring_stream_stride + hh * HD + slot * a.ring_slot_stride;
    for (int i = tid; i < 2 * CH; i += kRingThreads) {
      const int c = i % CH;
      if (i < CH)
        reinterpret_cast<uint4*>(kw)[c] = *reinterpret_cast<const uint4*>(sK + nvis * HD + c * 8);
      else
        reinterpret_cast<uint4*>(vw)[c] = *reinterpret_cast<const uint4*>(sV + nvis * HD + c * 8);
    }
  }
}

// One query frame, G heads per CTA, one warp per head: the streaming case with far fewer instructions per byte than
// ring_attn_frame_kernel (no block-wide barrier after the staging wait; every phase is warp-local). The G heads of a
// stream are contiguous in the ring rows and in q / k / v, so each ring row (distance d) of K and V for the group
// arrives by ONE bulk copy of G x HD halves (512 bytes for 4 x 64), all on one mbarrier, in distance order.
// Warp w = head hg * G + w: lane l scores keys l, l + 32, l + 64 (distance order, then the frame's own key) over 16-byte
// pieces in a rotated order (the 8 lanes of a quarter-warp read 8 distinct bank groups), fp16-rounded dot products
// scaled in fp32 (decoder_stream.py:172); the softmax runs in the warp, P rounded to fp16 (:173); lane l accumulates
// dims [l * HD / 32, (l + 1) * HD / 32) of P_ring.V_ring over the visible rows; o = fp16(fp16(ring) + fp16(p_self
// v_self)) (:174). Shared memory: K and V rows [nv + 1][G][HD], q [G][HD], P [G][nv + 1] floats, one mbarrier.
template <int HD, int G>
struct RingHeadsSmem {
  static constexpr int kRowHalves = G * HD;                  // one staged row: the G heads of one ring slot
  __host__ __device__ static size_t p_off(int nv) { return static_cast<size_t>(2 * (nv + 1) + 1) * kRowHalves * 2; }
  __host__ __device__ static size_t bar_off(int nv) { return (p_off(nv) + static_cast<size_t>(G) * (nv + 1) * 4 + 7) & ~size_t(7); }
  __host__ __device__ static size_t bytes(int nv) { return bar_off(nv) + 8; }
};

template <int HD, int G>
__global__ void __launch_bounds__(32 * G) ring_attn_frame_heads_kernel(const RingArgs a) {
  using SM = RingHeadsSmem<HD, G>;
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int CH = HD / 8;                                 // 16-byte pieces per head row
  constexpr int DPL = HD / 32;                               // output dims per lane (2 or 4)
  const int hg = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int RING = a.ring;
  const int NV = a.past < RING ? a.past : RING;              // ring rows any frame can see (launch-wide)
  __half* sK = reinterpret_cast<__half*>(smem);              // [NV + 1][G][HD]
  __half* sV = sK + (NV + 1) * SM::kRowHalves;
  __half* sQ = sV + (NV + 1) * SM::kRowHalves;               // [G][HD]
  float* sP = reinterpret_cast<float*>(smem + SM::p_off(NV)) + w * (NV + 1);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SM::bar_off(NV));

  const long long row = a.ring_rows[b];
  const long long pos = a.pos[b];
  const int pm1_mod = ring_pm1(pos, a);
  int nvis = NV;                                             // distance d lives in slot (pos-1-d) mod RING
  if (pos < nvis) nvis = pos < 0 ? 0 : static_cast<int>(pos);
  const int nk = nvis + 1;                                   // keys: nvis ring rows, then the frame itself
  constexpr uint32_t kRowBytes = SM::kRowHalves * sizeof(__half);

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(2 * nk + 1) * kRowBytes);
  }
  __syncthreads();
  const long long fo = b * a.qkv_batch_stride + hg * SM::kRowHalves;   // the frame's q / k / v rows of the group
  const __half* kr = a.k_ring + row * a.ring_stream_stride + hg * SM::kRowHalves;
  const __half* vr = a.v_ring + row * a.ring_stream_stride + hg * SM::kRowHalves;
  for (int i = tid; i < 2 * nk + 1; i += 32 * G) {
    const __half* src;
    __half* dst;
    if (i == 2 * nk) {
      src = a.q + fo;
      dst = sQ;
    } else {
      const int r = i >> 1;
      const bool v = (i & 1) != 0;
      if (r < nvis) {
        int j = pm1_mod - r;
        if (j < 0) j += RING;
        src = (v ? vr : kr) + j * a.ring_slot_stride;
      } else {
        src = (v ? a.v_new : a.k_new) + fo;
      }
      dst = (v ? sV : sK) + r * SM::kRowHalves;
    }
    bulk_g2s(dst, src, kRowBytes, bar);
  }
  if (!mbar_wait_bounded(bar, 0)) {
    // the copies did not land in time: flag it, keep the shared memory alive (bounded) until they are done, leave the
    // outputs untouched
    if (lane == 0) {
      atomicOr(a.status, kStatusWaitTimeout);
      mbar_wait_bounded(bar, 0, 100000000ull);
    }
    return;
  }

  // ---- scores of keys lane, lane + 32, ... : fp16-rounded dot products scaled in fp32
  const __half* qrow = sQ + w * HD;
  float sc[3];
  float m = -INFINITY;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    const int r = lane + 32 * u;
    sc[u] = -INFINITY;
    if (r < nk) {
      const __half* krow = sK + r * SM::kRowHalves + w * HD;
      float2 acc0 = make_float2(0.f, 0.f), acc1 = acc0;
#pragma unroll
      for (int pc = 0; pc < CH; ++pc) {
        const int pp = (pc + r) & (CH - 1);
        const uint4 kw = *reinterpret_cast<const uint4*>(krow + pp * 8);
        const uint4 qw = *reinterpret_cast<const uint4*>(qrow + pp * 8);
        const __half2* kh = reinterpret_cast<const __half2*>(&kw);
        const __half2* qh = reinterpret_cast<const __half2*>(&qw);
        acc0 = __ffma2_rn(__half22float2(kh[0]), __half22float2(qh[0]), acc0);
        acc1 = __ffma2_rn(__half22float2(kh[1]), __half22float2(qh[1]), acc1);
        acc0 = __ffma2_rn(__half22float2(kh[2]), __half22float2(qh[2]), acc0);
        acc1 = __ffma2_rn(__half22float2(kh[3]), __half22float2(qh[3]), acc1);
      }
      sc[u] = round_fp16((acc0.x + acc0.y) + (acc1.x + acc1.y)) * a.scale;
      m = fmaxf(m, sc[u]);
    }
  }
  m = warp_max(m);
  // ---- softmax in the warp, P rounded to fp16
  float e[3], sum = 0.f;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    e[u] = (lane + 32 * u < nk) ? expf(sc[u] - m) : 0.f;
    sum += e[u];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.f / sum;                               // the frame always sees itself: sum > 0
#pragma unroll
  for (int u = 0; u < 3; ++u)
    if (lane + 32 * u < nk) sP[lane + 32 * u] = round_fp16(e[u] * inv);
  __syncwarp();

  // ---- P_ring.V_ring: lane l owns DPL consecutive dims; o = fp16(fp16(ring) + fp16(p_self * v_self))
  const int d0 = lane * DPL;
  float acc[DPL];
#pragma unroll
  for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
  for (int r = 0; r < nvis; ++r) {
    const float pr = sP[r];
    const __half* vrow = sV + r * SM::kRowHalves + w * HD + d0;
    if constexpr (DPL == 2) {
      const float2 v2 = __half22float2(*reinterpret_cast<const __half2*>(vrow));
      acc[0] = fmaf(pr, v2.x, acc[0]);
      acc[1] = fmaf(pr, v2.y, acc[1]);
    } else {
      const uint2 vw = *reinterpret_cast<const uint2*>(vrow);
      const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vw.x));
      const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vw.y));
      acc[0] = fmaf(pr, v01.x, acc[0]);
      acc[1] = fmaf(pr, v01.y, acc[1]);
      acc[2] = fmaf(pr, v23.x, acc[2]);
      acc[3] = fmaf(pr, v23.y, acc[3]);
    }
  }
  const float pself = sP[nvis];
  const __half* vself = sV + nvis * SM::kRowHalves + w * HD + d0;
  __half* op = a.out + b * a.out_batch_stride + (hg * G + w) * HD + d0;
#pragma unroll
  for (int j = 0; j < DPL; j += 2) {
    const float2 vs = __half22float2(*reinterpret_cast<const __half2*>(vself + j));
    *reinterpret_cast<__half2*>(op + j) = __floats2half2_rn(round_fp16(acc[j]) + round_fp16(pself * vs.x),
                                                            round_fp16(acc[j + 1]) + round_fp16(pself * vs.y));
  }

  // ---- the frame's columns into the ring (a slot outside every window of this launch, never staged)
  if (a.write_new) {
    const int slot = ring_slot_after(pm1_mod, 0, RING);
    const long long off = row * a.ring_stream_stride + slot * a.ring_slot_stride + (hg * G + w) * HD + d0;
    const __half* ks = sK + nvis * SM::kRowHalves + w * HD + d0;
#pragma unroll
    for (int j = 0; j < DPL; j += 2) {
      *reinterpret_cast<__half2*>(a.k_ring + off + j) = *reinterpret_cast<const __half2*>(ks + j);
      *reinterpret_cast<__half2*>(a.v_ring + off + j) = *reinterpret_cast<const __half2*>(vself + j);
    }
  }
}

// One query frame on the tensor cores, G heads per CTA, one warp per head. The staging is that of
// ring_attn_frame_heads_kernel (ring rows of the G heads by distance, then the frame's row; one bulk copy per row),
// except that K (with q) and V complete on two mbarriers, so scores and softmax run while V lands, and that each
// staged row is padded by 16 bytes: the 8 rows an ldmatrix reads at one column offset then sit in 8 distinct bank
// groups. Per warp (head w), with the query as row 0 of a 16-row A operand (rows 1-15 zero):
//   S = q.K^T      mma.sync m16n8k16 over 8-key tiles, K fragments by ldmatrix.x4 (4 x 8 dims of 8 keys);
//   softmax        on the lanes holding row 0 (lanes 0-3, two keys per tile each): fp16-rounded scores scaled in
//                  fp32 (decoder_stream.py:172), P rounded to fp16 (:173);
//   O = P_ring.V   mma.sync over 16-key steps with P taken straight from the score fragments (a tile's C layout is
//                  the next contraction's A layout) and V fragments by ldmatrix.x4.trans; the frame's own key enters
//                  as fp16(p_self v_self) (:174).
// Key rows past the staged ones read a 16-byte zero row instead (ldmatrix takes one row address per lane), so no
// padding rows are copied or cleared, and a zero probability never meets stale shared memory.
template <int HD, int G>
struct RingMmaSmem {
  static constexpr int kRB = G * HD * 2;                     // bytes of a staged row: the G heads of one slot
  static constexpr int kRS = kRB + 16;                       // row stride in shared memory
  __host__ __device__ static size_t v_off(int nk) { return static_cast<size_t>(nk) * kRS; }
  __host__ __device__ static size_t q_off(int nk) { return 2 * static_cast<size_t>(nk) * kRS; }
  __host__ __device__ static size_t zero_off(int nk) { return q_off(nk) + kRB; }
  __host__ __device__ static size_t bar_off(int nk) { return zero_off(nk) + 16; }
  __host__ __device__ static size_t bytes(int nk) { return bar_off(nk) + 16; }
};



__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

constexpr int kRingMmaMaxKeys = 96;                          // key tiles of 8 held in registers: 12

// The tensor-core math of one query frame for one head (one warp), shared by the one-frame kernels: rows staged by
// distance at k_rows / v_rows (shared-memory addresses of this head's columns of row 0, rows rs bytes apart, the
// frame's own k / v as row nvis), q at q_head; keys past nvis read the 16-byte zero row at zero_addr. wait_v() is
// called after the softmax and before V is read (false: give up, nothing written). Writes the output row of
// (stream b, head) and, with write_new, the frame's k / v into ring slot pos % RING.
template <int HD, class WaitV>
__device__ __forceinline__ void ring_frame_head_mma(const RingArgs& a, uint32_t k_rows, uint32_t v_rows,
                                                    const uint8_t* q_head, const uint8_t* k_self, const uint8_t* v_self,
                                                    int rs, uint32_t zero_addr, int nvis, int b, int head,
                                                    long long row, long long pos, int lane, WaitV wait_v) {
  constexpr int NT = kRingMmaMaxKeys / 8;                    // score tiles (upper bound)
  constexpr int NTO = HD / 8;                                // output tiles of 8 dims
  const int t4 = lane & 3;
  const int RING = a.ring;
  const int nk = nvis + 1;
  const int nt = (nk + 7) >> 3;

  // ---- S = q.K^T on the tensor cores: A rows 1-15 are zero, so only lanes 0-3 carry q (row 0)
  uint32_t qa[HD / 16][2];
#pragma unroll
  for (int ks = 0; ks < HD / 16; ++ks) {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(q_head + ks * 32);
    qa[ks][0] = lane < 4 ? qw[t4] : 0u;                      // dims 16ks + 2t4, +1
    qa[ks][1] = lane < 4 ? qw[4 + t4] : 0u;                  // dims 16ks + 8 + 2t4, +1
  }
  float s[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    if (j < nt) {
      const int key = 8 * j + (lane & 7);
      const uint32_t ra = k_rows + key * rs + (lane >> 3) * 16;
#pragma unroll
      for (int kp = 0; kp < HD / 32; ++kp) {                 // 32 dims (two k-steps) per ldmatrix.x4
        uint32_t bf[4];
        ldsm_x4(key < nk ? ra + kp * 64 : zero_addr, bf);
        mma_f16(s[j], qa[2 * kp][0], 0u, qa[2 * kp][1], 0u, bf[0], bf[1]);
        mma_f16(s[j], qa[2 * kp + 1][0], 0u, qa[2 * kp + 1][1], 0u, bf[2], bf[3]);
      }
    }
  }

  // ---- softmax over row 0 (lanes 0-3 hold keys 8j + 2t4, +1 of every tile j); P rounded to fp16
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = 8 * j + 2 * t4 + e;
      const float x = (j < nt && key < nk) ? round_fp16(s[j][e]) * a.scale : -INFINITY;
      s[j][e] = x;
      m = fmaxf(m, x);
    }
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float x = (j < nt) ? expf(s[j][e] - m) : 0.f;   // masked keys: exp(-inf) = 0
      s[j][e] = x;
      sum += x;
    }
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  const float inv = 1.f / sum;                               // the frame always sees itself: sum > 0 (lanes 0-3)
  float pmine = 0.f;
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = 8 * j + 2 * t4 + e;
      float p = round_fp16(s[j][e] * inv);
      if (key == nvis) {                                     // the frame's own key: kept apart from the ring sum
        pmine = p;
        p = 0.f;
      }
      s[j][e] = lane < 4 ? p : 0.f;                          // rows 1-15 of the P operand are zero
    }
  const float pself = __shfl_sync(0xffffffffu, pmine, (nvis & 7) >> 1);

  if (!wait_v()) return;
  // ---- O_ring = P_ring.V_ring: 16-key steps; ldmatrix.x4.trans gives the V fragments of two 8-dim tiles
  float o[NTO][4];
#pragma unroll
  for (int jn = 0; jn < NTO; ++jn) o[jn][0] = o[jn][1] = o[jn][2] = o[jn][3] = 0.f;
  const int ksteps = (nk + 15) >> 4;
#pragma unroll
  for (int kk = 0; kk < NT / 2; ++kk) {
    if (kk < ksteps) {
      const uint32_t pa0 = pack_half2(s[2 * kk][0], s[2 * kk][1]);        // keys 16kk + 2t4, +1
      const uint32_t pa2 = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);  // keys 16kk + 8 + 2t4, +1
      const int key = 16 * kk + ((lane >> 3) & 1) * 8 + (lane & 7);
      const uint32_t ra = v_rows + key * rs + (lane >> 4) * 16;
#pragma unroll
      for (int np = 0; np < NTO / 2; ++np) {
        uint32_t bf[4];
        ldsm_x4_trans(key < nk ? ra + np * 32 : zero_addr, bf);
        mma_f16(o[2 * np], pa0, 0u, pa2, 0u, bf[0], bf[1]);
        mma_f16(o[2 * np + 1], pa0, 0u, pa2, 0u, bf[2], bf[3]);
      }
    }
  }

  // ---- o = fp16(fp16(ring) + fp16(p_self v_self)): lanes 0-3 hold dims 8jn + 2t4, +1
  if (lane < 4) {
    const __half* vself = reinterpret_cast<const __half*>(v_self);
    __half* op = a.out + b * a.out_batch_stride + head * HD;
#pragma unroll
    for (int jn = 0; jn < NTO; ++jn) {
      const int d = 8 * jn + 2 * t4;
      const float2 vs = __half22float2(*reinterpret_cast<const __half2*>(vself + d));
      *reinterpret_cast<__half2*>(op + d) = __floats2half2_rn(round_fp16(o[jn][0]) + round_fp16(pself * vs.x),
                                                              round_fp16(o[jn][1]) + round_fp16(pself * vs.y));
    }
  }

  // ---- the frame's columns into the ring (a slot outside every window of this launch, never staged)
  if (a.write_new) {
    constexpr int DPL = HD / 32;
    const int slot = ring_slot_after(ring_pm1(pos, a), 0, RING);
    const long long off = row * a.ring_stream_stride + slot * a.ring_slot_stride + head * HD + lane * DPL;
    const __half* ks = reinterpret_cast<const __half*>(k_self) + lane * DPL;
    const __half* vs = reinterpret_cast<const __half*>(v_self) + lane * DPL;
#pragma unroll
    for (int j = 0; j < DPL; j += 2) {
      *reinterpret_cast<__half2*>(a.k_ring + off + j) = *reinterpret_cast<const __half2*>(ks + j);
      *reinterpret_cast<__half2*>(a.v_ring + off + j) = *reinterpret_cast<const __half2*>(vs + j);
    }
  }
}

template <int HD, int G>
__global__ void __launch_bounds__(32 * G) ring_attn_frame_mma_kernel(const RingArgs a) {
  using SM = RingMmaSmem<HD, G>;
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int RB = SM::kRB, RS = SM::kRS;
  const int hg = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int RING = a.ring;
  const int NV = a.past < RING ? a.past : RING;              // ring rows any frame can see (launch-wide)
  uint8_t* sK = smem;
  uint8_t* sV = smem + SM::v_off(NV + 1);
  uint8_t* sQ = smem + SM::q_off(NV + 1);
  uint8_t* sZero = smem + SM::zero_off(NV + 1);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SM::bar_off(NV + 1));   // [0]: q and K rows, [1]: V rows

  const long long row = a.ring_rows[b];
  const long long pos = a.pos[b];
  const int pm1_mod = ring_pm1(pos, a);
  int nvis = NV;                                             // distance d lives in slot (pos-1-d) mod RING
  if (pos < nvis) nvis = pos < 0 ? 0 : static_cast<int>(pos);
  const int nk = nvis + 1;                                   // keys: nvis ring rows, then the frame itself

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bar[0], static_cast<uint32_t>(nk + 1) * RB);
    mbar_arrive_expect_tx(&bar[1], static_cast<uint32_t>(nk) * RB);
  }
  if (tid < 4) reinterpret_cast<uint32_t*>(sZero)[tid] = 0u;
  __syncthreads();
  const long long fo = b * a.qkv_batch_stride + hg * (G * HD);   // the frame's q / k / v rows of the group
  const __half* kr = a.k_ring + row * a.ring_stream_stride + hg * (G * HD);
  const __half* vr = a.v_ring + row * a.ring_stream_stride + hg * (G * HD);
  for (int i = tid; i < 2 * nk + 1; i += 32 * G) {           // q, then the K rows, then the V rows
    if (i == 0) {
      bulk_g2s(sQ, a.q + fo, RB, &bar[0]);
    } else {
      const bool v = i > nk;
      const int r = v ? i - 1 - nk : i - 1;
      const __half* src;
      if (r < nvis) {
        int j = pm1_mod - r;
        if (j < 0) j += RING;
        src = (v ? vr : kr) + j * a.ring_slot_stride;
      } else {
        src = (v ? a.v_new : a.k_new) + fo;
      }
      bulk_g2s((v ? sV : sK) + r * RS, src, RB, &bar[v ? 1 : 0]);
    }
  }
  auto give_up = [&]() {
    // the copies did not land in time: flag it, keep the shared memory alive (bounded) until they are done, leave
    // the outputs untouched
    if (lane == 0) {
      atomicOr(a.status, kStatusWaitTimeout);
      mbar_wait_bounded(&bar[0], 0, 100000000ull);
      mbar_wait_bounded(&bar[1], 0, 100000000ull);
    }
  };
  if (!mbar_wait_bounded(&bar[0], 0)) {
    give_up();
    return;
  }

  ring_frame_head_mma<HD>(a, smem_addr(sK) + w * HD * 2, smem_addr(sV) + w * HD * 2, sQ + w * HD * 2,
                          sK + nvis * RS + w * HD * 2, sV + nvis * RS + w * HD * 2, RS, smem_addr(sZero), nvis, b,
                          hg * G + w, row, pos, lane, [&]() -> bool {
                            if (mbar_wait_bounded(&bar[1], 0)) return true;
                            give_up();
                            return false;
                          });
}

// One query frame as a persistent TMA pipeline (head_dim 64). Each CTA walks (stream, head) items
// c, c + grid, c + 2 grid, ... with kTqQuads quads of four consumer warps, each quad fed by its own producer warp
// through a ring of kTqStages stages (full / empty mbarriers, one writer and one reader group per stage, so no phase
// can be overtaken). Quad q takes items q, q + kTqQuads, ... of the CTA in order.
//   * The producer stages an item with 2-D tensor boxes. The visible ring slots form one slot range, or two when the
//     window wraps the ring. Each range goes in as boxes of 8 slots x 64 dims (1 KB, 128-byte swizzle) for K and V,
//     so about 20 TMA operations instead of one bulk copy per row. q and the frame's own k / v come by 1-D bulk copies.
//     A box may run up to 7 slots past its range (other frames' slots, or zero fill past the ring's end); those rows
//     are masked out of the scores and read as the zero row by P.V, like every row outside the window.
//   * The four consumer warps split the item's keys by 16-key steps (warp w takes steps w, w + 4). They exchange the
//     row maximum, then the row sum, through shared memory, so P = fp16(exp(s - max) / sum) is rounded after the
//     whole row is normalised, as the reference's softmax-then-cast does (decoder_stream.py:172-173). Each warp's P.V
//     partial (fp32) is summed over the four warps before the fp16 rounding of the ring half (:173-175).
// One warp per item is latency-bound (a dependent chain of ldmatrix, mma and shuffles per key tile). Splitting the
// keys over a quad cuts that chain four-fold, and two CTAs per SM keep 20 warps resident. Loads of later items stream
// while earlier ones are computed, so DRAM sees no wave-wide gaps.
constexpr int kTqMaxKeys = 112;                              // staged rows + the frame's own key: 7 steps of 16

struct RingTmaHeader {
  long long row, pos;
  int b, head;
  int n1, r2, n2;                                            // rows [0, n1) and [r2, r2 + n2) hold visible slots
  int seg1, seg2;                                            // ... slots [seg1, seg1 + n1) and [seg2, seg2 + n2)
  int pm1;                                                   // (pos - 1) mod RING: the newest frame's slot
};

// Rows per range are rounded up to 8 (one box), so two ranges of nvis <= NV rows together need floor8(NV + 14) rows.
__host__ __device__ inline int tma_stage_rows(int nv) { return ((nv + 14) / 8) * 8; }

template <int NQ, int NS, int NF = 1>
struct RingTmaSmem {
  static constexpr int kRowBytes = 128;                      // 64 fp16 dims
  __host__ __device__ static size_t v_off(int kr) { return static_cast<size_t>(kr) * kRowBytes; }
  // q rows [0, NF), the chunk's k rows [NF, 2 NF), its v rows [2 NF, 3 NF)
  __host__ __device__ static size_t self_off(int kr) { return 2 * static_cast<size_t>(kr) * kRowBytes; }
  __host__ __device__ static size_t hdr_off(int kr) { return self_off(kr) + 3 * NF * kRowBytes; }
  __host__ __device__ static size_t stage_bytes(int kr) {
    return (hdr_off(kr) + sizeof(RingTmaHeader) + 1023) & ~static_cast<size_t>(1023);
  }
  // per quad, one frame: row maxima [4], row sums [4], p_self, a give-up snapshot (index 9), then the four warps' P.V
  // partials [4][64]; a chunk: row maxima [4][8], row sums [4][8], the snapshot (index 64) (its P.V partials go to the
  // stage's K region)
  static constexpr size_t kXBytes = NF == 1 ? 64 + 4 * 64 * 4 : 512;
  static constexpr int kFlag = NF == 1 ? 9 : 64;
  __host__ __device__ static size_t x_off(int kr) { return NQ * NS * stage_bytes(kr); }
  __host__ __device__ static size_t zero_off(int kr) { return x_off(kr) + NQ * kXBytes; }
  __host__ __device__ static size_t flag_off(int kr) { return zero_off(kr) + 16; }
  __host__ __device__ static size_t bar_off(int kr) { return flag_off(kr) + 16; }   // full[quads][stages], then empty
  __host__ __device__ static size_t bytes(int kr) { return bar_off(kr) + 2 * NQ * NS * 8 + 1024; }
  static constexpr int kThreads = 32 * NQ * 5;               // a producer warp and four consumers per quad
};

struct RingTmaParams {
  RingArgs a;
  CUtensorMap km, vm;                                        // {64 dims, heads, slots, stream rows} of the K / V rings
};

__device__ __forceinline__ void quad_sync(int quad) {
  asm volatile("bar.sync %0, 128;" ::"r"(1 + quad) : "memory");
}

// One consumer warp's share of an item: 16-key steps wq and wq + 4 of the staged rows (K / V regions at k_reg / v_reg,
// 1024-aligned, 128-byte rows swizzled by row & 7; the frame's own key is key kr, its k / v unswizzled in `self`).
// The quad's four warps meet at three barriers per item: row maximum, row sum, P.V partials. `ok` is false after a
// give-up: the warp still takes part in every barrier, but writes nothing outside shared memory.
__device__ __forceinline__ void ring_tma_quad_math(const RingArgs& a, uint32_t k_reg, uint32_t v_reg,
                                                   const uint8_t* self, int kr, uint32_t zero_addr,
                                                   const RingTmaHeader& hd, float* xch, int quad, int wq, int lane,
                                                   bool ok) {
  constexpr int HD = 64;
  constexpr int NTO = HD / 8;
  const int t4 = lane & 3;
  const int nsteps = (kr + 1 + 15) >> 4;                     // 16-key steps over the staged rows and the own key
  const uint32_t self_addr = smem_addr(self);
  auto visible_row = [&](int key) -> bool {
    return key < kr && (key < hd.n1 || (key >= hd.r2 && key < hd.r2 + hd.n2));
  };

  uint32_t qa[HD / 16][2];
#pragma unroll
  for (int ks = 0; ks < HD / 16; ++ks) {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(self + ks * 32);
    qa[ks][0] = lane < 4 ? qw[t4] : 0u;
    qa[ks][1] = lane < 4 ? qw[4 + t4] : 0u;
  }
  // ---- scores of this warp's steps (two 8-key tiles each), masked, fp16-rounded and scaled
  float s[2][2][4];
  float m = -INFINITY;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int kk = wq + 4 * u;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      s[u][t][0] = s[u][t][1] = s[u][t][2] = s[u][t][3] = 0.f;
      if (kk < nsteps) {
        const int key = 16 * kk + 8 * t + (lane & 7);
#pragma unroll
        for (int kp = 0; kp < HD / 32; ++kp) {
          const int c = kp * 4 + (lane >> 3);
          const uint32_t addr = key < kr ? k_reg + key * 128 + ((c ^ (key & 7)) << 4)
                                         : (key == kr ? self_addr + 128 + c * 16 : zero_addr);
          uint32_t bf[4];
          ldsm_x4(addr, bf);
          mma_f16(s[u][t], qa[2 * kp][0], 0u, qa[2 * kp][1], 0u, bf[0], bf[1]);
          mma_f16(s[u][t], qa[2 * kp + 1][0], 0u, qa[2 * kp + 1][1], 0u, bf[2], bf[3]);
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = 16 * kk + 8 * t + 2 * t4 + e;
        const bool vis = kk < nsteps && (key == kr || visible_row(key));
        const float x = vis ? round_fp16(s[u][t][e]) * a.scale : -INFINITY;
        s[u][t][e] = x;
        m = fmaxf(m, x);
      }
    }
  }
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  if (lane == 0) xch[wq] = m;
  quad_sync(quad);                                           // (1) row maxima
  const float M = fmaxf(fmaxf(xch[0], xch[1]), fmaxf(xch[2], xch[3]));   // the own key is always visible: finite
  float sum = 0.f;
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float x = s[u][t][e] == -INFINITY ? 0.f : expf(s[u][t][e] - M);
        s[u][t][e] = x;
        sum += x;
      }
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  if (lane == 0) xch[4 + wq] = sum;
  quad_sync(quad);                                           // (2) row sums
  const float inv = 1.f / (((xch[4] + xch[5]) + xch[6]) + xch[7]);
  // ---- P = fp16(e / sum); the own key's probability kept apart from the ring sum
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = 16 * (wq + 4 * u) + 8 * t + 2 * t4 + e;
        float p = round_fp16(s[u][t][e] * inv);
        if (key == kr) {
          if (lane < 4) xch[8] = p;                          // one lane of one warp holds it
          p = 0.f;
        }
        s[u][t][e] = lane < 4 ? p : 0.f;
      }
  // ---- this warp's P.V partial over its steps; rows without a visible slot read the zero row
  float o[NTO][4];
#pragma unroll
  for (int jn = 0; jn < NTO; ++jn) o[jn][0] = o[jn][1] = o[jn][2] = o[jn][3] = 0.f;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int kk = wq + 4 * u;
    if (kk < nsteps) {
      const uint32_t pa0 = pack_half2(s[u][0][0], s[u][0][1]);
      const uint32_t pa2 = pack_half2(s[u][1][0], s[u][1][1]);
      const int key = 16 * kk + ((lane >> 3) & 1) * 8 + (lane & 7);
      const bool vis = visible_row(key);
#pragma unroll
      for (int np = 0; np < NTO / 2; ++np) {
        const int c = np * 2 + (lane >> 4);
        uint32_t bf[4];
        ldsm_x4_trans(vis ? v_reg + key * 128 + ((c ^ (key & 7)) << 4) : zero_addr, bf);
        mma_f16(o[2 * np], pa0, 0u, pa2, 0u, bf[0], bf[1]);
        mma_f16(o[2 * np + 1], pa0, 0u, pa2, 0u, bf[2], bf[3]);
      }
    }
  }
  float* part = xch + 16;                                    // [warp][64]
  if (lane < 4) {
#pragma unroll
    for (int jn = 0; jn < NTO; ++jn) {
      part[wq * 64 + 8 * jn + 2 * t4] = o[jn][0];
      part[wq * 64 + 8 * jn + 2 * t4 + 1] = o[jn][1];
    }
  }
  quad_sync(quad);                                           // (3) partials
  // ---- warp wq writes dims 16 wq .. 16 wq + 15: o = fp16(fp16(sum of partials) + fp16(p_self v_self))
  if (lane < 16 && ok) {
    const int d = 16 * wq + lane;
    const float ring = ((part[d] + part[64 + d]) + part[128 + d]) + part[192 + d];
    const float vs = __half2float(reinterpret_cast<const __half*>(self + 256)[d]);
    a.out[hd.b * a.out_batch_stride + hd.head * HD + d] = __float2half_rn(round_fp16(ring) + round_fp16(xch[8] * vs));
  }
  if (wq == 0 && ok && a.write_new) {
    const int RING = a.ring;
    const int slot = ring_slot_after(hd.pm1, 0, RING);
    const long long off = hd.row * a.ring_stream_stride + slot * a.ring_slot_stride + hd.head * HD + lane * 2;
    *reinterpret_cast<__half2*>(a.k_ring + off) = *reinterpret_cast<const __half2*>(self + 128 + lane * 4);
    *reinterpret_cast<__half2*>(a.v_ring + off) = *reinterpret_cast<const __half2*>(self + 256 + lane * 4);
  }
}

// One consumer warp's share of a chunk of n = 2 .. NF frames (rows 0 .. n-1 of the A operand; q, the chunk's k and
// v rows unswizzled in `self` at rows [0, NF), [NF, 2 NF), [2 NF, 3 NF)). Ring steps wq and wq + 4 as in
// ring_tma_quad_math; warp 3 also takes the chunk's own keys as one extra 8-key tile. Per row i: a ring row at
// distance d is visible when it holds a window slot and d <= past - 1 - i (decoder_stream.py:152-155), the chunk's key
// jj when jj <= i (:156). Row maxima and sums are exchanged through xch ([4][8] each); the P.V partials (ring:
// [4 warps][NF rows][64], chunk: [NF][64] fp32) go to `part`, the stage's K region, free once the scores are read.
// o = fp16(fp16(sum of ring partials) + fp16(chunk partial)) (:173-175).
template <int NF>
__device__ __forceinline__ void ring_tma_chunk_math(const RingArgs& a, uint32_t k_reg, uint32_t v_reg,
                                                    const uint8_t* self, float* part, int kr, uint32_t zero_addr,
                                                    const RingTmaHeader& hd, float* xch, int quad, int wq, int lane,
                                                    bool ok) {
  constexpr int HD = 64;
  constexpr int NTO = HD / 8;
  const int n = a.n, g = lane >> 2, t4 = lane & 3;
  const int RING = a.ring, PAST = a.past;
  const int nrs = (kr + 15) >> 4;                            // 16-key steps over the staged ring rows
  const uint32_t self_addr = smem_addr(self);
  auto visible_row = [&](int key) -> bool {
    return key < kr && (key < hd.n1 || (key >= hd.r2 && key < hd.r2 + hd.n2));
  };
  auto dist = [&](int key) -> int {                          // distance back from the newest frame of a visible row
    const int slot = key < hd.n1 ? hd.seg1 + key : hd.seg2 + (key - hd.r2);
    const int d = hd.pm1 - slot;
    return d < 0 ? d + RING : d;
  };

  // ---- Q fragments: rows 0 .. n-1 of the A operand
  uint32_t qa[HD / 16][4];
  {
    const int qr = ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks)
      ldsm_x4(qr < n ? self_addr + qr * 128 + (ks * 2 + (lane >> 4)) * 16 : zero_addr, qa[ks]);
  }
  // ---- scores: ring steps wq, wq + 4, and (warp 3) the chunk's keys; only row g (< n <= 8) is real in each lane
  float s[2][2][4], sn[4] = {0.f, 0.f, 0.f, 0.f};
  float m = -INFINITY;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int kk = wq + 4 * u;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      s[u][t][0] = s[u][t][1] = s[u][t][2] = s[u][t][3] = 0.f;
      if (kk < nrs) {
        const int key = 16 * kk + 8 * t + (lane & 7);
#pragma unroll
        for (int kp = 0; kp < HD / 32; ++kp) {
          const int c = kp * 4 + (lane >> 3);
          uint32_t bf[4];
          ldsm_x4(key < kr ? k_reg + key * 128 + ((c ^ (key & 7)) << 4) : zero_addr, bf);
          mma_f16(s[u][t], qa[2 * kp][0], qa[2 * kp][1], qa[2 * kp][2], qa[2 * kp][3], bf[0], bf[1]);
          mma_f16(s[u][t], qa[2 * kp + 1][0], qa[2 * kp + 1][1], qa[2 * kp + 1][2], qa[2 * kp + 1][3], bf[2], bf[3]);
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = 16 * kk + 8 * t + 2 * t4 + e;
        const bool vis = kk < nrs && g < n && visible_row(key) && dist(key) <= PAST - 1 - g;
        const float x = vis ? round_fp16(s[u][t][e]) * a.scale : -INFINITY;
        s[u][t][e] = x;
        m = fmaxf(m, x);
      }
    }
  }
  if (wq == 3) {
    const int jj = lane & 7;                                 // the chunk's key this lane addresses
#pragma unroll
    for (int kp = 0; kp < HD / 32; ++kp) {
      const int c = kp * 4 + (lane >> 3);
      uint32_t bf[4];
      ldsm_x4(jj < n ? self_addr + (NF + jj) * 128 + c * 16 : zero_addr, bf);
      mma_f16(sn, qa[2 * kp][0], qa[2 * kp][1], qa[2 * kp][2], qa[2 * kp][3], bf[0], bf[1]);
      mma_f16(sn, qa[2 * kp + 1][0], qa[2 * kp + 1][1], qa[2 * kp + 1][2], qa[2 * kp + 1][3], bf[2], bf[3]);
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = 2 * t4 + e;
      const bool vis = g < n && key < n && key <= g;
      const float x = vis ? round_fp16(sn[e]) * a.scale : -INFINITY;
      sn[e] = x;
      m = fmaxf(m, x);
    }
  }
  // ---- row maxima and sums across the quad (lanes 4g .. 4g+3 hold row g)
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  if (t4 == 0) xch[wq * 8 + g] = m;
  quad_sync(quad);                                           // (1) row maxima
  const float M = fmaxf(fmaxf(xch[g], xch[8 + g]), fmaxf(xch[16 + g], xch[24 + g]));
  float sum = 0.f;
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float x = s[u][t][e] == -INFINITY ? 0.f : expf(s[u][t][e] - M);
        s[u][t][e] = x;
        sum += x;
      }
  if (wq == 3) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float x = sn[e] == -INFINITY ? 0.f : expf(sn[e] - M);
      sn[e] = x;
      sum += x;
    }
  }
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  if (t4 == 0) xch[32 + wq * 8 + g] = sum;
  quad_sync(quad);                                           // (2) row sums
  const float L = ((xch[32 + g] + xch[40 + g]) + xch[48 + g]) + xch[56 + g];
  const float inv = L > 0.f ? 1.f / L : 0.f;                 // rows past n have no key
#pragma unroll
  for (int u = 0; u < 2; ++u)
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) s[u][t][e] = round_fp16(s[u][t][e] * inv);
  sn[0] = round_fp16(sn[0] * inv);
  sn[1] = round_fp16(sn[1] * inv);

  // ---- ring P.V partial over this warp's steps (rows without a visible slot read the zero row)
  float o[NTO][4];
#pragma unroll
  for (int jn = 0; jn < NTO; ++jn) o[jn][0] = o[jn][1] = o[jn][2] = o[jn][3] = 0.f;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int kk = wq + 4 * u;
    if (kk < nrs) {
      const uint32_t pa0 = pack_half2(s[u][0][0], s[u][0][1]);
      const uint32_t pa2 = pack_half2(s[u][1][0], s[u][1][1]);
      const int key = 16 * kk + ((lane >> 3) & 1) * 8 + (lane & 7);
      const bool vis = visible_row(key);
#pragma unroll
      for (int np = 0; np < NTO / 2; ++np) {
        const int c = np * 2 + (lane >> 4);
        uint32_t bf[4];
        ldsm_x4_trans(vis ? v_reg + key * 128 + ((c ^ (key & 7)) << 4) : zero_addr, bf);
        mma_f16(o[2 * np], pa0, 0u, pa2, 0u, bf[0], bf[1]);
        mma_f16(o[2 * np + 1], pa0, 0u, pa2, 0u, bf[2], bf[3]);
      }
    }
  }
  if (g < n) {
#pragma unroll
    for (int jn = 0; jn < NTO; ++jn) {
      part[(wq * NF + g) * 64 + 8 * jn + 2 * t4] = o[jn][0];
      part[(wq * NF + g) * 64 + 8 * jn + 2 * t4 + 1] = o[jn][1];
    }
  }
  // ---- the chunk's P.V (warp 3): one 16-key step over its v rows, keys past n read the zero row
  if (wq == 3) {
#pragma unroll
    for (int jn = 0; jn < NTO; ++jn) o[jn][0] = o[jn][1] = o[jn][2] = o[jn][3] = 0.f;
    const uint32_t pa0 = pack_half2(sn[0], sn[1]);
    const int key = ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int np = 0; np < NTO / 2; ++np) {
      const int c = np * 2 + (lane >> 4);
      uint32_t bf[4];
      ldsm_x4_trans(key < n ? self_addr + (2 * NF + key) * 128 + c * 16 : zero_addr, bf);
      mma_f16(o[2 * np], pa0, 0u, 0u, 0u, bf[0], bf[1]);
      mma_f16(o[2 * np + 1], pa0, 0u, 0u, 0u, bf[2], bf[3]);
    }
    if (g < n) {
#pragma unroll
      for (int jn = 0; jn < NTO; ++jn) {
        part[(4 * NF + g) * 64 + 8 * jn + 2 * t4] = o[jn][0];
        part[(4 * NF + g) * 64 + 8 * jn + 2 * t4 + 1] = o[jn][1];
      }
    }
  }
  quad_sync(quad);                                           // (3) partials
  // ---- warp wq writes dims 16 wq .. 16 wq + 15 of every row
  if (lane < 16 && ok) {
    const int d = 16 * wq + lane;
    for (int i = 0; i < n; ++i) {
      const float ring = ((part[i * 64 + d] + part[(NF + i) * 64 + d]) + part[(2 * NF + i) * 64 + d]) +
                         part[(3 * NF + i) * 64 + d];
      const float own = part[(4 * NF + i) * 64 + d];
      a.out[hd.b * a.out_batch_stride + i * a.out_frame_stride + hd.head * HD + d] =
          __float2half_rn(round_fp16(ring) + round_fp16(own));
    }
  }
  // ---- the chunk's k / v into ring slots (pos + jj) % RING
  if (ok && a.write_new) {
    for (int jj = wq; jj < n; jj += 4) {
      const int slot = ring_slot_after(hd.pm1, jj, RING);
      const long long off = hd.row * a.ring_stream_stride + slot * a.ring_slot_stride + hd.head * HD + lane * 2;
      *reinterpret_cast<__half2*>(a.k_ring + off) = *reinterpret_cast<const __half2*>(self + (NF + jj) * 128 + lane * 4);
      *reinterpret_cast<__half2*>(a.v_ring + off) =
          *reinterpret_cast<const __half2*>(self + (2 * NF + jj) * 128 + lane * 4);
    }
  }
  fence_proxy_async_smem();                                  // `part` (generic stores) is the next item's TMA target
}

template <int NQ, int NS, int MINB, int NF>
__global__ void __launch_bounds__(32 * NQ * 5, MINB) ring_attn_frame_tma_kernel(const __grid_constant__ RingTmaParams P) {
  using SMEM = RingTmaSmem<NQ, NS, NF>;
  constexpr int kTqQuads = NQ, kTqStages = NS;
  const RingArgs& a = P.a;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // 128-byte swizzled boxes need 1024-byte aligned destinations: align the dynamic shared memory base at run time
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int RING = a.ring;
  const int NV = a.past < RING ? a.past : RING;              // ring rows any frame can see (launch-wide)
  const int kr = tma_stage_rows(NV);
  const size_t SB = SMEM::stage_bytes(kr);
  uint8_t* sZero = smem + SMEM::zero_off(kr);
  volatile int* abort_flag = reinterpret_cast<int*>(smem + SMEM::flag_off(kr));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SMEM::bar_off(kr));   // [quad * kTqStages + stage]
  uint64_t* empty = full + NQ * NS;
  const long long items = static_cast<long long>(a.B) * a.H;
  const long long nloc = (items - blockIdx.x + gridDim.x - 1) / gridDim.x;   // this CTA's items (grid <= items)
  const int nf = NF == 1 ? 1 : a.n;                          // frames of the chunk (1 .. NF)

  if (tid == 0) {
    for (int i = 0; i < NQ * NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (tid < 4) reinterpret_cast<uint32_t*>(sZero)[tid] = 0u;
  __syncthreads();

  if (warp < kTqQuads) {
    // ---- producer of quad `warp`: items warp, warp + kTqQuads, ... of this CTA
    const int quad = warp;
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.km)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.vm)) : "memory");
    }
    long long j = 0;
    long long nrow = 0, npos = 0;
    if (quad < nloc) {
      const int b0 = static_cast<int>((blockIdx.x + static_cast<long long>(quad) * gridDim.x) / a.H);
      nrow = a.ring_rows[b0];
      npos = a.pos[b0];
    }
    for (long long k = quad; k < nloc; k += kTqQuads, ++j) {
      const long long item = blockIdx.x + k * gridDim.x;
      const int b = static_cast<int>(item / a.H), head = static_cast<int>(item % a.H);
      const long long row = nrow, pos = npos;
      if (k + kTqQuads < nloc) {                             // the next item's ring row and position, loaded early
        const int bn = static_cast<int>((item + static_cast<long long>(kTqQuads) * gridDim.x) / a.H);
        nrow = a.ring_rows[bn];
        npos = a.pos[bn];
      }
      const int bi = quad * kTqStages + static_cast<int>(j % kTqStages);
      if (j >= kTqStages && !mbar_wait_bounded(&empty[bi], static_cast<uint32_t>((j / kTqStages - 1) & 1))) {
        if (lane == 0) {
          atomicOr(a.status, kStatusWaitTimeout);
          *abort_flag = 1;
        }
      }
      __syncwarp();
      if (*abort_flag) break;
      // visible slots: distances 0 .. nvis-1 back from slot pm1 = (pos - 1) mod RING, i.e. slots
      // [pm1 - nvis + 1, pm1], or [0, pm1] and [RING - (nvis - pm1 - 1), RING) when that wraps
      const int pm1_mod = ring_pm1(pos, a);
      int nvis = NV;
      if (pos < nvis) nvis = pos < 0 ? 0 : static_cast<int>(pos);
      const int s_lo = pm1_mod - nvis + 1;
      int seg1 = 0, n1 = nvis, seg2 = 0, n2 = 0;
      if (s_lo >= 0) {
        seg1 = s_lo;
      } else {
        n1 = pm1_mod + 1;
        seg2 = RING + s_lo;
        n2 = -s_lo;
      }
      const int r2 = (n1 + 7) & ~7;
      const int nb1 = (n1 + 7) >> 3, nb2 = (n2 + 7) >> 3, nb = nb1 + nb2;
      uint8_t* S = smem + bi * SB;
      if (lane == 0) {
        RingTmaHeader* h = reinterpret_cast<RingTmaHeader*>(S + SMEM::hdr_off(kr));
        h->row = row;
        h->pos = pos;
        h->b = b;
        h->head = head;
        h->n1 = n1;
        h->r2 = r2;
        h->n2 = n2;
        h->seg1 = seg1;
        h->seg2 = seg2;
        h->pm1 = pm1_mod;
        mbar_arrive_expect_tx(&full[bi], static_cast<uint32_t>(2 * nb) * 1024u + static_cast<uint32_t>(3 * nf) * 128u);
      }
      __syncwarp();
      const uint32_t sa = smem_addr(S), bar = smem_addr(&full[bi]);
      const long long fo = b * a.qkv_batch_stride + head * 64;
      for (int i = lane; i < 3 * nf + 2 * nb; i += 32) {
        if (i < 3 * nf) {                                    // q, then the chunk's k, then its v rows
          const int kind = i / nf, f = i - kind * nf;
          const __half* src = (kind == 0 ? a.q : (kind == 1 ? a.k_new : a.v_new)) + fo + f * a.qkv_frame_stride;
          bulk_g2s(S + SMEM::self_off(kr) + (kind * NF + f) * 128, src, 128, &full[bi]);
        } else {
          const int t = i - 3 * nf, kv = t >= nb ? 1 : 0, bx = t - kv * nb;
          const int slot = bx < nb1 ? seg1 + 8 * bx : seg2 + 8 * (bx - nb1);
          const int r = bx < nb1 ? 8 * bx : r2 + 8 * (bx - nb1);
          tma_load_4d(sa + static_cast<uint32_t>(kv ? SMEM::v_off(kr) : 0) + r * 128, kv ? &P.vm : &P.km, 0,
                      head, slot, static_cast<int>(row), bar);
        }
      }
    }
    const long long mine = (nloc - quad + kTqQuads - 1) / kTqQuads;
    if (j < mine && lane == 0) {
      // gave up: the stages issued last may still be landing; wait for them (bounded) before the CTA can exit
      for (long long jj = j > kTqStages ? j - kTqStages : 0; jj < j; ++jj)
        mbar_wait_bounded(&full[quad * kTqStages + static_cast<int>(jj % kTqStages)],
                          static_cast<uint32_t>((jj / kTqStages) & 1), 100000000ull);
    }
    return;
  }

  // ---- consumer warp wq of quad `quad`; every warp of a quad takes the same barriers, item after item, even after
  //      a give-up (then writing nothing outside shared memory), and the quad leaves together
  const int quad = (warp - kTqQuads) >> 2, wq = (warp - kTqQuads) & 3;
  float* xch = reinterpret_cast<float*>(smem + SMEM::x_off(kr) + quad * SMEM::kXBytes);
  const uint32_t zero_addr = smem_addr(sZero);
  long long j = 0;
  for (long long k = quad; k < nloc; k += kTqQuads, ++j) {
    const int bi = quad * kTqStages + static_cast<int>(j % kTqStages);
    if (!mbar_wait_bounded(&full[bi], static_cast<uint32_t>((j / kTqStages) & 1))) {
      if (lane == 0) {
        atomicOr(a.status, kStatusWaitTimeout);
        *abort_flag = 1;
      }
    }
    __syncwarp();
    const bool ok = *abort_flag == 0;
    const uint8_t* S = smem + bi * SB;
    const RingTmaHeader hd = *reinterpret_cast<const RingTmaHeader*>(S + SMEM::hdr_off(kr));
    const uint32_t sa = smem_addr(S);
    if constexpr (NF == 1)
      ring_tma_quad_math(a, sa, sa + static_cast<uint32_t>(SMEM::v_off(kr)), S + SMEM::self_off(kr), kr, zero_addr,
                         hd, xch, quad, wq, lane, ok);
    else
      ring_tma_chunk_math<NF>(a, sa, sa + static_cast<uint32_t>(SMEM::v_off(kr)), S + SMEM::self_off(kr),
                              reinterpret_cast<float*>(smem + bi * SB), kr, zero_addr, hd, xch, quad, wq, lane, ok);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[bi]);
    // one snapshot of the give-up flag per item, taken by warp 0 before the barrier, so all four warps of the quad
    // break after the same item (the flag itself may change at any time)
    if (wq == 0 && lane == 0) xch[SMEM::kFlag] = *abort_flag ? 1.f : 0.f;
    quad_sync(quad);
    if (xch[SMEM::kFlag] != 0.f) break;
  }
}

// A chunk of 2 .. 16 frames on the tensor cores, G heads per CTA, one warp per head: the design of
// ring_attn_frame_mma_kernel with the n query rows as rows 0 .. n-1 of the A operand (Q fragments by ldmatrix.x4 from
// padded rows, rows past n read the zero row). Each lane holds rows g and g + 8 of every score tile and applies the
// row's own mask in registers: ring row d is visible to query i when d < nvis and d <= past - 1 - i
// (decoder_stream.py:152-155), the chunk's key jj when jj <= i (:156). The two halves of the output are two tensor-core
// passes over the same V fragments, P restricted to the ring keys, then to the chunk's keys, each rounded to fp16
// before the sum (:173-175).
template <int HD, int G>
struct RingChunkSmem {
  static constexpr int kRB = G * HD * 2;                     // bytes of a staged row: the G heads of one slot / frame
  static constexpr int kRS = kRB + 16;                       // row stride in shared memory (bank-group rotation)
  __host__ __device__ static size_t v_off(int nk) { return static_cast<size_t>(nk) * kRS; }
  __host__ __device__ static size_t q_off(int nk) { return 2 * static_cast<size_t>(nk) * kRS; }
  __host__ __device__ static size_t zero_off(int nk, int n) { return q_off(nk) + static_cast<size_t>(n) * kRS; }
  __host__ __device__ static size_t bar_off(int nk, int n) { return zero_off(nk, n) + 16; }
  __host__ __device__ static size_t bytes(int nk, int n) { return bar_off(nk, n) + 16; }
};

constexpr int kRingChunkMaxKeys = 112;                       // ring rows + chunk keys held as score tiles: 14 x 8
constexpr int kRingChunkMaxFrames = 16;                      // one 16-row query tile

template <int HD, int G>
__global__ void __launch_bounds__(32 * G) ring_attn_chunk_mma_kernel(const RingArgs a) {
  using SM = RingChunkSmem<HD, G>;
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int RB = SM::kRB, RS = SM::kRS;
  constexpr int NT = kRingChunkMaxKeys / 8;                  // score tiles (upper bound)
  constexpr int NTO = HD / 8;                                // output tiles of 8 dims
  const int hg = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int n = a.n, RING = a.ring, PAST = a.past;
  const int NV = PAST < RING ? PAST : RING;                  // ring rows any frame can see (launch-wide)
  const int NKL = NV + n;
  uint8_t* sK = smem;
  uint8_t* sV = smem + SM::v_off(NKL);
  uint8_t* sQ = smem + SM::q_off(NKL);
  uint8_t* sZero = smem + SM::zero_off(NKL, n);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SM::bar_off(NKL, n));   // [0]: q and K rows, [1]: V rows

  const long long row = a.ring_rows[b];
  const long long pos = a.pos[b];
  const int pm1_mod = ring_pm1(pos, a);
  int nvis = NV;                                             // distance d lives in slot (pos-1-d) mod RING
  if (pos < nvis) nvis = pos < 0 ? 0 : static_cast<int>(pos);
  const int nk = nvis + n;                                   // keys: nvis ring rows, then the chunk's n frames

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bar[0], static_cast<uint32_t>(n + nk) * RB);
    mbar_arrive_expect_tx(&bar[1], static_cast<uint32_t>(nk) * RB);
  }
  if (tid < 4) reinterpret_cast<uint32_t*>(sZero)[tid] = 0u;
  __syncthreads();
  const long long fo = b * a.qkv_batch_stride + hg * (G * HD);   // frame 0's q / k / v rows of the group
  const __half* kr = a.k_ring + row * a.ring_stream_stride + hg * (G * HD);
  const __half* vr = a.v_ring + row * a.ring_stream_stride + hg * (G * HD);
  for (int i = tid; i < n + 2 * nk; i += 32 * G) {           // the q rows, then the K rows, then the V rows
    if (i < n) {
      bulk_g2s(sQ + i * RS, a.q + fo + i * a.qkv_frame_stride, RB, &bar[0]);
    } else {
      const bool v = i >= n + nk;
      const int r = v ? i - n - nk : i - n;
      const __half* src;
      if (r < nvis) {
        int j = pm1_mod - r;
        if (j < 0) j += RING;
        src = (v ? vr : kr) + j * a.ring_slot_stride;
      } else {
        src = (v ? a.v_new : a.k_new) + fo + (r - nvis) * a.qkv_frame_stride;
      }
      bulk_g2s((v ? sV : sK) + r * RS, src, RB, &bar[v ? 1 : 0]);
    }
  }
  auto give_up = [&]() {
    if (lane == 0) {
      atomicOr(a.status, kStatusWaitTimeout);
      mbar_wait_bounded(&bar[0], 0, 100000000ull);
      mbar_wait_bounded(&bar[1], 0, 100000000ull);
    }
  };
  if (!mbar_wait_bounded(&bar[0], 0)) {
    give_up();
    return;
  }

  const uint32_t zero_addr = smem_addr(sZero);
  const uint32_t k_base = smem_addr(sK) + w * HD * 2;
  const uint32_t v_base = smem_addr(sV) + w * HD * 2;
  const int nt = (nk + 7) >> 3;

  // ---- Q fragments (rows 0 .. n-1 real) for every 16-dim step
  uint32_t qa[HD / 16][4];
  {
    const int qr = ((lane >> 3) & 1) * 8 + (lane & 7);
    const uint32_t qaddr = smem_addr(sQ) + qr * RS + w * HD * 2 + (lane >> 4) * 16;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) ldsm_x4(qr < n ? qaddr + ks * 32 : zero_addr, qa[ks]);
  }
  // ---- S = Q.K^T
  float s[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    if (j < nt) {
      const int key = 8 * j + (lane & 7);
      const uint32_t ra = k_base + key * RS + (lane >> 3) * 16;
#pragma unroll
      for (int kp = 0; kp < HD / 32; ++kp) {
        uint32_t bf[4];
        ldsm_x4(key < nk ? ra + kp * 64 : zero_addr, bf);
        mma_f16(s[j], qa[2 * kp][0], qa[2 * kp][1], qa[2 * kp][2], qa[2 * kp][3], bf[0], bf[1]);
        mma_f16(s[j], qa[2 * kp + 1][0], qa[2 * kp + 1][1], qa[2 * kp + 1][2], qa[2 * kp + 1][3], bf[2], bf[3]);
      }
    }
  }

  // ---- masked softmax of rows g (elements 0, 1) and g + 8 (elements 2, 3) across the lane quad; P rounded to fp16
  float m[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = g + (e >> 1) * 8, c = 8 * j + 2 * t4 + (e & 1);
      const bool ok = j < nt && i < n && c < nk && (c < nvis ? c <= PAST - 1 - i : c - nvis <= i);
      const float x = ok ? round_fp16(s[j][e]) * a.scale : -INFINITY;
      s[j][e] = x;
      m[e >> 1] = fmaxf(m[e >> 1], x);
    }
  float sum[2];
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    m[h2] = fmaxf(m[h2], __shfl_xor_sync(0xffffffffu, m[h2], 1));
    m[h2] = fmaxf(m[h2], __shfl_xor_sync(0xffffffffu, m[h2], 2));
    sum[h2] = 0.f;
  }
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x = s[j][e] == -INFINITY ? 0.f : expf(s[j][e] - m[e >> 1]);   // rows past n: all masked
      s[j][e] = x;
      sum[e >> 1] += x;
    }
  float inv[2];
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    sum[h2] += __shfl_xor_sync(0xffffffffu, sum[h2], 1);
    sum[h2] += __shfl_xor_sync(0xffffffffu, sum[h2], 2);
    inv[h2] = sum[h2] > 0.f ? 1.f / sum[h2] : 0.f;           // a real query always sees itself
  }
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[j][e] = round_fp16(s[j][e] * inv[e >> 1]);

  if (!mbar_wait_bounded(&bar[1], 0)) {
    give_up();
    return;
  }
  // ---- O_ring = P_ring.V over the 16-key steps holding ring rows, then O_new = P_new.V over those holding the chunk's
  //      keys; the same ldmatrix.x4.trans V fragments, P restricted by key index
  float o[NTO][4];
  uint32_t oring[NTO][2];                                    // fp16(O_ring), rows g and g + 8
  const int ks_ring = (nvis + 15) >> 4, ks_first_new = nvis >> 4, ks_end = (nk + 15) >> 4;
#pragma unroll
  for (int pass = 0; pass < 2; ++pass) {
#pragma unroll
    for (int jn = 0; jn < NTO; ++jn) o[jn][0] = o[jn][1] = o[jn][2] = o[jn][3] = 0.f;
    const int k_lo = pass == 0 ? 0 : ks_first_new, k_hi = pass == 0 ? ks_ring : ks_end;
#pragma unroll
    for (int kk = 0; kk < NT / 2; ++kk) {
      if (kk >= k_lo && kk < k_hi) {
        uint32_t pa[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {                        // a0a1: row g, keys +2t4; a2a3: row g+8; a4..a7: keys +8
          const int j = 2 * kk + (r >> 1), e0 = (r & 1) * 2;
          const int c = 8 * j + 2 * t4;
          const bool in0 = pass == 0 ? c < nvis : c >= nvis, in1 = pass == 0 ? c + 1 < nvis : c + 1 >= nvis;
          pa[r] = pack_half2(in0 ? s[j][e0] : 0.f, in1 ? s[j][e0 + 1] : 0.f);
        }
        const int key = 16 * kk + ((lane >> 3) & 1) * 8 + (lane & 7);
        const uint32_t ra = v_base + key * RS + (lane >> 4) * 16;
#pragma unroll
        for (int np = 0; np < NTO / 2; ++np) {
          uint32_t bf[4];
          ldsm_x4_trans(key < nk ? ra + np * 32 : zero_addr, bf);
          mma_f16(o[2 * np], pa[0], pa[1], pa[2], pa[3], bf[0], bf[1]);
          mma_f16(o[2 * np + 1], pa[0], pa[1], pa[2], pa[3], bf[2], bf[3]);
        }
      }
    }
    if (pass == 0) {
#pragma unroll
      for (int jn = 0; jn < NTO; ++jn) {
        oring[jn][0] = pack_half2(o[jn][0], o[jn][1]);
        oring[jn][1] = pack_half2(o[jn][2], o[jn][3]);
      }
    }
  }
  // ---- o = fp16(fp16(O_ring) + fp16(O_new)) for rows g, g + 8 below n
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    const int i = g + 8 * h2;
    if (i < n) {
      __half* op = a.out + b * a.out_batch_stride + i * a.out_frame_stride + (hg * G + w) * HD + 2 * t4;
#pragma unroll
      for (int jn = 0; jn < NTO; ++jn) {
        const float2 r = __half22float2(*reinterpret_cast<const __half2*>(&oring[jn][h2]));
        *reinterpret_cast<__half2*>(op + 8 * jn) =
            __floats2half2_rn(r.x + round_fp16(o[jn][2 * h2]), r.y + round_fp16(o[jn][2 * h2 + 1]));
      }
    }
  }

  // ---- the chunk's columns into ring slots (pos + jj) % RING (outside every window of this launch, never staged)
  if (a.write_new) {
    constexpr int DPL = HD / 32;
    for (int jj = 0; jj < n; ++jj) {
      const int slot = ring_slot_after(pm1_mod, jj, RING);
      const long long off = row * a.ring_stream_stride + slot * a.ring_slot_stride + (hg * G + w) * HD + lane * DPL;
      const __half* ks = reinterpret_cast<const __half*>(sK + (nvis + jj) * RS) + w * HD + lane * DPL;
      const __half* vs = reinterpret_cast<const __half*>(sV + (nvis + jj) * RS) + w * HD + lane * DPL;
#pragma unroll
      for (int j = 0; j < DPL; j += 2) {
        *reinterpret_cast<__half2*>(a.k_ring + off + j) = *reinterpret_cast<const __half2*>(ks + j);
        *reinterpret_cast<__half2*>(a.v_ring + off + j) = *reinterpret_cast<const __half2*>(vs + j);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------------
// One query frame with nothing staged (selection 6): each (stream, head) is one CTA of W warps (4 for head_dim 64, 8
// for 128), and every K and V row the frame sees goes straight from HBM into registers, all loads issued before the
// first is used. A row takes LPR = head_dim / 8 lanes (16 bytes each), so a warp load reads RG = 32 / LPR whole rows
// (four of 128 bytes or two of 256). Warp w holds key rows r = RG (W i + w) + g, i < P + R (distance order; the
// frame's own key is row nvis), lane l = LPR g + c the piece c (dims 8c .. 8c+7) of them; a lane keeps (P + R) x 2
// pieces in flight.
//   scores   per-lane partial dot products over 8 dims (fp32), completed over the LPR lanes of a row group by a
//            transposing butterfly in a batch of P rows and one of R (afterwards lane c holds the score of batch index
//            c / (LPR / P), resp. P + c / (LPR / R)); fp16-rounded, scaled in fp32 (decoder_stream.py:172);
//   softmax  each warp's (max, sum of exp) pair meets the others' in shared memory, so every warp normalises with the
//            whole row's max and sum before P is rounded to fp16 (:173);
//   P.V      each lane takes its rows' probabilities by shuffles and accumulates its 8 dims; the RG row groups meet by
//            a second transposing butterfly (lane (g, c) ends with the DPL = 8 / RG dims 8c + DPL g ..), warps 1 .. W-1
//            hand their partial sums (and p_self) to warp 0 through shared memory; o = fp16(fp16(ring) + fp16(p_self
//            v_self)) (:174).
// Measured at head_dim 64 against one warp per (stream, head) (18 rows per lane group, 168 registers), 2, 6 and 8
// warps per item, and a resident grid walking the items: four warps per item, one item per CTA, at nine CTAs per SM
// gave the shortest layer (the number of items in flight per SM is what counts).
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t ld_nc_u1(const void* p) {
  uint32_t r;
  asm("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

// Sum the N per-lane values v (N a power of two, at most LPR) over the LPR lanes of a lane group (xor offsets LPR / 2
// .. 1; LPR 8 or 16); the result is the complete sum of value index c / (LPR / N), c = lane % LPR.
template <int N, int LPR>
__device__ __forceinline__ float group_transpose_sum(float (&v)[N], int c) {
  static_assert(N >= 1 && N <= LPR && (N & (N - 1)) == 0 && (LPR == 8 || LPR == 16), "N a power of two <= LPR");
  int off = LPR / 2;
#pragma unroll
  for (int n = N; n > 1; n >>= 1, off >>= 1) {
    const bool up = (c & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = up ? v[i] : v[i + n / 2];
      const float keep = up ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  float s = v[0];
#pragma unroll
  for (; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  return s;
}

// 8 fp16 of a 16-byte piece dotted with 8 fp32 (two chains of packed FMAs)
__device__ __forceinline__ float dot8_h(const uint4 w, const float2 (&q)[4]) {
  const __half2* h = reinterpret_cast<const __half2*>(&w);
  float2 a0 = __fmul2_rn(__half22float2(h[0]), q[0]);
  float2 a1 = __fmul2_rn(__half22float2(h[1]), q[1]);
  a0 = __ffma2_rn(__half22float2(h[2]), q[2], a0);
  a1 = __ffma2_rn(__half22float2(h[3]), q[3], a1);
  return (a0.x + a0.y) + (a1.x + a1.y);
}

// Warps per (stream, head): head_dim 64 rows take 8 lanes (four rows per warp load), 128 take 16 (two rows), so 4 / 8
// warps keep 5 rows per lane group either way.
__host__ __device__ constexpr int ring_stream_warps(int hd) { return hd == 64 ? 4 : 8; }
constexpr int kRingStreamRows = 5;                           // rows per lane group and warp: P + R = 4 + 1
constexpr int kRingStreamMaxKeys = 80;                       // ring rows + the frame's own key: (32 / LPR) W * 5

template <int HD>
__global__ void __launch_bounds__(32 * ring_stream_warps(HD)) ring_attn_frame_stream_kernel(const RingArgs a) {
  constexpr int W = ring_stream_warps(HD), P = 4, R = 1, RPL = P + R;
  constexpr int LPR = HD / 8, RG = 32 / LPR, DPL = 8 / RG;   // lanes per row, row groups per warp, output dims per lane
  static_assert(RPL == kRingStreamRows && RG * W * RPL == kRingStreamMaxKeys, "row batches");
  constexpr int SP = LPR / P, SR = LPR / R;                  // lanes holding one completed score of a batch
  using SelfW = typename std::conditional<DPL == 2, uint32_t, uint2>::type;   // DPL halves of the frame's k / v
  __shared__ float2 s_ml[W];                                 // (max, sum of exp(s - max)) per warp
  __shared__ float s_acc[W - 1][DPL + 1][32];                // warps 1 .. W-1: DPL output dims and p_self per lane
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane / LPR, c = lane % LPR;
  const int b = static_cast<int>(blockIdx.x / a.H), head = static_cast<int>(blockIdx.x % a.H);   // grid = B * H
  const int RING = a.ring;
  const int NV = a.past < RING ? a.past : RING;              // ring rows any frame can see (launch-wide)
  const long long row = a.ring_rows[b];
  const long long pos = a.pos[b];
  const int pm1_mod = ring_pm1_mod(pos, RING, a.ring_magic, a.ring_shift);   // distance d: slot (pos-1-d) mod RING
  int nvis = NV;
  if (pos < nvis) nvis = pos < 0 ? 0 : static_cast<int>(pos);
  const int nk = nvis + 1;                                   // <= kRingStreamMaxKeys (checked by the launcher)

  // ---- every load, K first: ring rows by distance and the frame's own key; V of the ring rows only (the frame's own
  //      value enters through p_self)
  const long long fo = b * a.qkv_batch_stride + head * HD;   // the frame's q / k / v row of this head
  const long long ro = row * a.ring_stream_stride + head * HD + c * 8;
  const int d0 = 8 * c + DPL * g;                            // the DPL output dims of this lane
  const uint4 qw = ld_stream_v4(a.q + fo + c * 8);
  SelfW vself_w{}, kself_w{};
  if (w == 0) {
    if constexpr (DPL == 2) {
      vself_w = ld_nc_u1(a.v_new + fo + d0);
      if (a.write_new) kself_w = ld_nc_u1(a.k_new + fo + d0);
    } else {
      vself_w = ld_nc_u2(a.v_new + fo + d0);
      if (a.write_new) kself_w = ld_nc_u2(a.k_new + fo + d0);
    }
  }
  uint4 kw[RPL], vw[RPL];
#pragma unroll
  for (int i = 0; i < RPL; ++i) {
    const int r = RG * (W * i + w) + g;
    kw[i] = make_uint4(0u, 0u, 0u, 0u);
    if (r < nvis) {
      int j = pm1_mod - r;
      if (j < 0) j += RING;
      kw[i] = ld_stream_v4(a.k_ring + ro + j * a.ring_slot_stride);
    } else if (r == nvis) {
      kw[i] = ld_stream_v4(a.k_new + fo + c * 8);
    }
  }
#pragma unroll
  for (int i = 0; i < RPL; ++i) {
    const int r = RG * (W * i + w) + g;
    vw[i] = make_uint4(0u, 0u, 0u, 0u);
    if (r < nvis) {
      int j = pm1_mod - r;
      if (j < 0) j += RING;
      vw[i] = ld_stream_v4(a.v_ring + ro + j * a.ring_slot_stride);
    }
  }

  // ---- scores
  float2 q2[4];
  {
    const __half2* qh = reinterpret_cast<const __half2*>(&qw);
#pragma unroll
    for (int j = 0; j < 4; ++j) q2[j] = __half22float2(qh[j]);
  }
  float s[2];
  {
    float part[P];
#pragma unroll
    for (int i = 0; i < P; ++i) part[i] = dot8_h(kw[i], q2);
    s[0] = group_transpose_sum<P, LPR>(part, c);
    float rest[R];
#pragma unroll
    for (int i = 0; i < R; ++i) rest[i] = dot8_h(kw[P + i], q2);
    s[1] = group_transpose_sum<R, LPR>(rest, c);
  }
  const int rr[2] = {RG * (W * (c / SP) + w) + g, RG * (W * (P + c / SR) + w) + g};
  const bool first[2] = {(c % SP) == 0, (c % SR) == 0};      // the lane that counts a duplicated score once
  float mw = -INFINITY;
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    s[u] = rr[u] < nk ? round_fp16(s[u]) * a.scale : -INFINITY;
    mw = fmaxf(mw, s[u]);
  }
  mw = warp_max(mw);
  float lw = 0.f;
#pragma unroll
  for (int u = 0; u < 2; ++u) lw += (rr[u] < nk && first[u]) ? expf(s[u] - mw) : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
  // ---- the row's max and sum over the W warps (a warp with no visible key reports (-inf, 0))
  if (lane == 0) s_ml[w] = make_float2(mw, lw);
  __syncthreads();
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < W; ++j) m = fmaxf(m, s_ml[j].x);       // finite: the frame's own key is in some warp
  float l = 0.f;
#pragma unroll
  for (int j = 0; j < W; ++j) l += s_ml[j].y > 0.f ? s_ml[j].y * expf(s_ml[j].x - m) : 0.f;
  const float inv = 1.f / l;
  float p[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) p[u] = rr[u] < nk ? round_fp16(expf(s[u] - m) * inv) : 0.f;
  // p_self, on the warp holding row nvis = RG (W i_s + w_s) + g_s
  const int qd = nvis / RG, w_s = qd % W, i_s = qd / W, g_s = nvis % RG;
  float pself = 0.f;
  if (w == w_s)
    pself = __shfl_sync(0xffffffffu, i_s < P ? p[0] : p[1], LPR * g_s + (i_s < P ? i_s * SP : (i_s - P) * SR));

  // ---- P_ring.V_ring over this lane's rows (V of rows >= nvis is zero), then over the row groups and the warps
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
  for (int i = 0; i < RPL; ++i) {
    const float pi = i < P ? __shfl_sync(0xffffffffu, p[0], LPR * g + i * SP)
                           : __shfl_sync(0xffffffffu, p[1], LPR * g + (i - P) * SR);
    const float2 pp = make_float2(pi, pi);
    const __half2* vh = reinterpret_cast<const __half2*>(&vw[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 t = make_float2(acc[2 * j], acc[2 * j + 1]);
      t = __ffma2_rn(__half22float2(vh[j]), pp, t);
      acc[2 * j] = t.x;
      acc[2 * j + 1] = t.y;
    }
  }
  // transposing butterfly over the row groups (xor 16 .. LPR): lane (g, c) ends with dims 8c + DPL g .. + DPL - 1
#pragma unroll
  for (int n = 8, off = 16; off >= LPR; n >>= 1, off >>= 1) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = up ? acc[i] : acc[i + n / 2];
      const float keep = up ? acc[i + n / 2] : acc[i];
      acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  if (w > 0) {
#pragma unroll
    for (int j = 0; j < DPL; ++j) s_acc[w - 1][j][lane] = acc[j];
    s_acc[w - 1][DPL][lane] = pself;
  }
  __syncthreads();
  if (w > 0) return;
#pragma unroll
  for (int k = 0; k < W - 1; ++k) {
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] += s_acc[k][j][lane];
    pself += s_acc[k][DPL][lane];
  }
  const __half2* vsh = reinterpret_cast<const __half2*>(&vself_w);
  __half2 ov[DPL / 2];
#pragma unroll
  for (int j = 0; j < DPL / 2; ++j) {
    const float2 vs = __half22float2(vsh[j]);
    ov[j] = __floats2half2_rn(round_fp16(acc[2 * j]) + round_fp16(pself * vs.x),
                              round_fp16(acc[2 * j + 1]) + round_fp16(pself * vs.y));
  }
  __half2* op = reinterpret_cast<__half2*>(a.out + b * a.out_batch_stride + head * HD + d0);   // 4-byte aligned
#pragma unroll
  for (int j = 0; j < DPL / 2; ++j) op[j] = ov[j];
  // ---- the frame's columns into the ring (a slot outside every window of this launch, never loaded)
  if (a.write_new) {
    const int pos_mod = pm1_mod + 1 == RING ? 0 : pm1_mod + 1;
    const long long off = row * a.ring_stream_stride + pos_mod * a.ring_slot_stride + head * HD + d0;
    *reinterpret_cast<SelfW*>(a.k_ring + off) = kself_w;
    *reinterpret_cast<SelfW*>(a.v_ring + off) = vself_w;
  }
}

static size_t frame_smem_bytes(int ring, int past, int hd) {
  const int nv = past < ring ? past : ring;
  return static_cast<size_t>(2 * (nv + 1) + 1) * hd * sizeof(__half) + static_cast<size_t>((nv + 1 + 3) & ~3) * 4 +
         static_cast<size_t>(kRingThreads / 32) * hd * 4 + sizeof(uint64_t);
}

size_t ring_smem_bytes(int ring, int past, int hd, int n) { return RingGeom(ring, past, n).bytes(hd, n); }

int g_ring_frame_kernel = 6;

// ceil(2^(63 + l) / d) and l - 1, l = ceil(log2 d), for ring_pm1_mod (2 <= d <= kRingMaxSlots)
static void ring_reciprocal(int d, unsigned long long* magic, int* shift) {
  int l = 1;
  while ((1 << l) < d) ++l;
  const unsigned __int128 num = static_cast<unsigned __int128>(1) << (63 + l);
  *magic = static_cast<unsigned long long>((num + static_cast<unsigned>(d) - 1u) / static_cast<unsigned>(d));
  *shift = l - 1;
}
int g_ring_chunk_kernel = 1;

// The pipelined TMA one-frame kernel: head_dim 64, stage rings that fit the SM's shared memory, row strides in whole
// 16-byte units (tensor maps), and a driver that offers the tensor-map encoder. Otherwise *launched stays false.
static bool make_ring_map(CUtensorMap* m, const void* base, const RingArgs& a) {
  const EncodeTiled enc = tensor_map_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || (a.ring_slot_stride * 2) % 16 ||
      (a.ring_stream_stride * 2) % 16 || a.ring_slot_stride <= 0 || a.ring_stream_stride <= 0)
    return false;
  // the stream-row extent is not part of the call: the largest row coordinate a map can take, never reached
  const cuuint64_t dims[4] = {64u, static_cast<cuuint64_t>(a.H), static_cast<cuuint64_t>(a.ring), 0x7fffffffu};
  const cuuint64_t strides[3] = {128u, static_cast<cuuint64_t>(a.ring_slot_stride) * 2,
                                 static_cast<cuuint64_t>(a.ring_stream_stride) * 2};
  const cuuint32_t box[4] = {64u, 1u, 8u, 1u};
  const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NQ, int NS, int MINB, int NF>
static cudaError_t launch_frame_tma_cfg(int nv, const RingArgs& a, cudaStream_t stream, bool* launched) {
  using SMEM = RingTmaSmem<NQ, NS, NF>;
  *launched = false;
  const int kr = tma_stage_rows(nv);
  if (a.hd != 64 || kr + 1 > kTqMaxKeys || SMEM::bytes(kr) * MINB > 227u * 1024u) return cudaSuccess;
  // a chunk: 2 .. NF frames, and the stage's K region must hold the P.V partials ([5 NF][64] fp32)
  if (NF > 1 && (a.n < 2 || a.n > NF || static_cast<size_t>(kr) * 128 < static_cast<size_t>(5 * NF) * 64 * 4))
    return cudaSuccess;
  RingTmaParams p;
  memset(&p, 0, sizeof(p));
  p.a = a;
  if (!make_ring_map(&p.km, a.k_ring, a) || !make_ring_map(&p.vm, a.v_ring, a)) return cudaSuccess;
  static thread_local int sm_dev = -1, sms = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (sm_dev != dev) {
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(ring_attn_frame_tma_kernel<NQ, NS, MINB, NF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(227u * 1024u / MINB));
    if (e != cudaSuccess) return e;
    sm_dev = dev;
  }
  const long long items = static_cast<long long>(a.B) * a.H;
  const long long slots = static_cast<long long>(MINB) * sms;
  const int grid = static_cast<int>(items < slots ? items : slots);
  ring_attn_frame_tma_kernel<NQ, NS, MINB, NF><<<grid, 32 * NQ * 5, SMEM::bytes(kr), stream>>>(p);
  *launched = true;
  return cudaGetLastError();
}

// Two quads of two stages, two CTAs per SM: measured against three quads of three stages and two quads of four
// stages at one CTA per SM (24.2-24.6 against 27.6-27.9 and 32.6 us per layer at 256 streams x 16 heads).
static cudaError_t launch_frame_tma(int nv, const RingArgs& a, cudaStream_t stream, bool* launched) {
  return launch_frame_tma_cfg<2, 2, 2, 1>(nv, a, stream, launched);
}

static cudaError_t launch_chunk_tma(int nv, const RingArgs& a, cudaStream_t stream, bool* launched) {
  return launch_frame_tma_cfg<2, 2, 2, 8>(nv, a, stream, launched);
}

template <int HD, int G>
static cudaError_t set_mma_frame_smem() {
  return cudaFuncSetAttribute(ring_attn_frame_mma_kernel<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(RingMmaSmem<HD, G>::bytes(kRingMmaMaxKeys)));
}

template <int HD, int G>
static cudaError_t launch_mma_frame(dim3 grid, int nv, const RingArgs& a, cudaStream_t stream) {
  ring_attn_frame_mma_kernel<HD, G><<<grid, 32 * G, RingMmaSmem<HD, G>::bytes(nv + 1), stream>>>(a);
  return cudaGetLastError();
}

template <int HD, int G>
static cudaError_t set_chunk_smem() {
  return cudaFuncSetAttribute(ring_attn_chunk_mma_kernel<HD, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(RingChunkSmem<HD, G>::bytes(kRingChunkMaxKeys, kRingChunkMaxFrames)));
}

template <int HD, int G>
static cudaError_t launch_chunk(dim3 grid, int nv, const RingArgs& a, cudaStream_t stream) {
  ring_attn_chunk_mma_kernel<HD, G><<<grid, 32 * G, RingChunkSmem<HD, G>::bytes(nv + a.n, a.n), stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ring_attn(const RingArgs& args, cudaStream_t stream) {
  RingArgs a = args;                                         // + the ring's reciprocal for the kernels' slot arithmetic
  if (a.ring >= 2) ring_reciprocal(a.ring, &a.ring_magic, &a.ring_shift);
  // the shared-memory limits are raised once per device, for the largest ring and chunk supported, so a call made
  // during stream capture sets no attribute
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    const int m64 = static_cast<int>(ring_smem_bytes(kRingMaxSlots, kRingMaxSlots, 64, kRingMaxChunk));
    const int m128 = static_cast<int>(ring_smem_bytes(kRingMaxSlots, kRingMaxSlots, 128, kRingMaxChunk));
    const int s64 = static_cast<int>(frame_smem_bytes(kRingMaxSlots, kRingMaxSlots, 64));
    const int s128 = static_cast<int>(frame_smem_bytes(kRingMaxSlots, kRingMaxSlots, 128));
    cudaError_t e = cudaFuncSetAttribute(ring_attn_mma_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, m64);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(ring_attn_mma_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, m128);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(ring_attn_frame_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, s64);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(ring_attn_frame_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, s128);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(ring_attn_frame_heads_kernel<64, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(RingHeadsSmem<64, 4>::bytes(95)));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(ring_attn_frame_heads_kernel<128, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(RingHeadsSmem<128, 2>::bytes(95)));
    if (e == cudaSuccess) e = set_mma_frame_smem<64, 4>();
    if (e == cudaSuccess) e = set_mma_frame_smem<64, 2>();
    if (e == cudaSuccess) e = set_mma_frame_smem<64, 1>();
    if (e == cudaSuccess) e = set_mma_frame_smem<128, 2>();
    if (e == cudaSuccess) e = set_mma_frame_smem<128, 1>();
    if (e == cudaSuccess) e = set_chunk_smem<64, 4>();
    if (e == cudaSuccess) e = set_chunk_smem<64, 2>();
    if (e == cudaSuccess) e = set_chunk_smem<64, 1>();
    if (e == cudaSuccess) e = set_chunk_smem<128, 2>();
    if (e == cudaSuccess) e = set_chunk_smem<128, 1>();
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  if (a.B == 0 || a.n == 0) return cudaSuccess;
  const int nv = a.past < a.ring ? a.past : a.ring;
  if (a.n == 1 && g_ring_frame_kernel == 5) {
    bool launched = false;
    const cudaError_t e = launch_frame_tma(nv, a, stream, &launched);
    if (e != cudaSuccess || launched) return e;
  }
  if (a.n == 1 && nv < kRingMmaMaxKeys) {
    // one frame on the tensor cores, G heads per CTA: 4 x 64 or 2 x 128 halves per staged row (selection 0; 3 and 4
    // take fewer heads per CTA); under 75 KB of shared memory per CTA at 71 visible rows, so three CTAs per SM
    const int sel = g_ring_frame_kernel;
    if (sel == 0 || sel == 3 || sel == 4) {
      const int G = sel == 4 ? 1 : (sel == 3 ? (a.hd == 64 ? 2 : 1) : (a.hd == 64 ? 4 : 2));
      if (a.H % G == 0) {
        const dim3 mgrid(a.H / G, a.B);
        if (a.hd == 64) {
          if (G == 4) return launch_mma_frame<64, 4>(mgrid, nv, a, stream);
          if (G == 2) return launch_mma_frame<64, 2>(mgrid, nv, a, stream);
          return launch_mma_frame<64, 1>(mgrid, nv, a, stream);
        }
        if (G == 2) return launch_mma_frame<128, 2>(mgrid, nv, a, stream);
        return launch_mma_frame<128, 1>(mgrid, nv, a, stream);
      }
    }
  }
  if (a.n >= 2 && g_ring_chunk_kernel == 4) {
    bool launched = false;
    const cudaError_t e = launch_chunk_tma(nv, a, stream, &launched);
    if (e != cudaSuccess || launched) return e;
  }
  if (a.n >= 2 && a.n <= kRingChunkMaxFrames && nv + a.n <= kRingChunkMaxKeys && g_ring_chunk_kernel != 1 &&
      g_ring_chunk_kernel != 4) {
    // 2 .. 16 frames on the tensor cores, G heads per CTA: 2 x 64 / 1 x 128 (selection 0), 4 x 64 / 2 x 128 (2),
    // one head (3)
    const int sel = g_ring_chunk_kernel;
    const int G = sel == 3 ? 1 : (sel == 2 ? (a.hd == 64 ? 4 : 2) : (a.hd == 64 ? 2 : 1));
    if (a.H % G == 0) {
      const dim3 cgrid(a.H / G, a.B);
      if (a.hd == 64) {
        if (G == 4) return launch_chunk<64, 4>(cgrid, nv, a, stream);
        if (G == 2) return launch_chunk<64, 2>(cgrid, nv, a, stream);
        return launch_chunk<64, 1>(cgrid, nv, a, stream);
      }
      if (G == 2) return launch_chunk<128, 2>(cgrid, nv, a, stream);
      return launch_chunk<128, 1>(cgrid, nv, a, stream);
    }
  }
  if (a.n == 1 && g_ring_frame_kernel == 6 && a.ring >= 2 && nv + 1 <= kRingStreamMaxKeys &&
      static_cast<long long>(a.B) * a.H <= 2147483647ll) {
    // one frame, nothing staged: a CTA of 4 (head_dim 64) or 8 (128) warps per (stream, head)
    const unsigned items = static_cast<unsigned>(static_cast<long long>(a.B) * a.H);
    if (a.hd == 64)
      ring_attn_frame_stream_kernel<64><<<items, 32 * ring_stream_warps(64), 0, stream>>>(a);
    else
      ring_attn_frame_stream_kernel<128><<<items, 32 * ring_stream_warps(128), 0, stream>>>(a);
    return cudaGetLastError();
  }
  if (a.n == 1 && (g_ring_frame_kernel == 2 || g_ring_frame_kernel == 6) && nv <= 95) {
    // one frame, scalar math, G heads per CTA (4 x 64 or 2 x 128 halves per staged row); also the calls selection 6
    // does not fit (head_dim 128, wider windows)
    const int G = a.hd == 64 ? 4 : 2;
    if (a.H % G == 0) {
      const dim3 hgrid(a.H / G, a.B);
      if (a.hd == 64) {
        const size_t bytes = RingHeadsSmem<64, 4>::bytes(nv);
        ring_attn_frame_heads_kernel<64, 4><<<hgrid, 128, bytes, stream>>>(a);
      } else {
        const size_t bytes = RingHeadsSmem<128, 2>::bytes(nv);
        ring_attn_frame_heads_kernel<128, 2><<<hgrid, 64, bytes, stream>>>(a);
      }
      return cudaGetLastError();
    }
  }
  dim3 grid(a.B, a.H);
  if (a.n == 1) {
    const size_t bytes = frame_smem_bytes(a.ring, a.past, a.hd);
    if (a.hd == 64)
      ring_attn_frame_kernel<64><<<grid, kRingThreads, bytes, stream>>>(a);
    else
      ring_attn_frame_kernel<128><<<grid, kRingThreads, bytes, stream>>>(a);
  } else {
    const size_t bytes = ring_smem_bytes(a.ring, a.past, a.hd, a.n);
    if (a.hd == 64)
      ring_attn_mma_kernel<64><<<grid, kRingThreads, bytes, stream>>>(a);
    else
      ring_attn_mma_kernel<128><<<grid, kRingThreads, bytes, stream>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace q3
