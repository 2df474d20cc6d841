// Pieces shared by the paged decode kernels (paged_decode.cu: CUDA-core scoring; paged_decode_mma.cu: warp MMA
// scoring): the flat split-K plan, the seat/chunk cursor, the chunk copy descriptors and the end-of-seat
// write / partial / merge. paged_decode.cu describes the work distribution.
#pragma once
#include "q3_common.cuh"
#include "q3_kernels.h"

namespace q3 {

constexpr int kDecodeWarps = kKvHeads;             // one warp per KV head
constexpr int kDecodeThreads = kDecodeWarps * 32;  // 256

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

// The chunk split. Uniform: CTA c of Ge takes [c*N/Ge, (c+1)*N/Ge). Pair-weighted (H > 0, Ge = 2H CTAs, two per SM):
// the CTAs a block index below H (the first to become resident on each SM) take kPairW1 shares and the others
// kPairW2: the younger CTA of an SM gets fewer issue slots, so equal shares leave it finishing last. With
// S(c) = W1*c (c <= H) or W1*H + W2*(c - H), CTA c takes [N*S(c)/T, N*S(c+1)/T), T = S(Ge).
constexpr int kPairW1 = 47, kPairW2 = 45;

__device__ __forceinline__ long long pair_share(int c, int H) {
  return c <= H ? static_cast<long long>(kPairW1) * c
                : static_cast<long long>(kPairW1) * H + static_cast<long long>(kPairW2) * (c - H);
}

// First chunk of CTA c.
__device__ __forceinline__ long long chunk_start(int c, long long N, int Ge, int H) {
  if (H == 0) return (N * c) / Ge;
  return (N * pair_share(c, H)) / pair_share(Ge, H);
}

// CTA index owning global chunk p: the largest c whose first chunk is <= p.
__device__ __forceinline__ int cta_of_chunk(long long p, long long N, int Ge, int H) {
  if (H == 0) return static_cast<int>(((p + 1) * Ge + N - 1) / N - 1);
  const long long X = ((p + 1) * pair_share(Ge, H) - 1) / N;   // chunk_start(c) <= p  <=>  S(c) <= X
  const long long c = X < static_cast<long long>(kPairW1) * H ? X / kPairW1
                                                                 : H + (X - static_cast<long long>(kPairW1) * H) / kPairW2;
  return static_cast<int>(c < Ge - 1 ? c : Ge - 1);
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

// What the copies of one chunk need. Built one iteration before the chunk is issued, so the block-table load in it
// has landed by the time the (last-reading) warp issues the copies.
struct ChunkDesc {
  long long row0;   // pool row of the chunk's first token when the chunk lies in one page, else -1
  int seat, tok0, rows, pool_rows;
  bool has_new;
};

template <int ROWS>
__device__ __forceinline__ ChunkDesc make_desc(const DecodeArgs& a, const SeatCursor& cur, long long i) {
  ChunkDesc d;
  d.seat = cur.seat;
  d.tok0 = static_cast<int>(i - cur.first) * ROWS;
  d.rows = min(ROWS, cur.len - d.tok0);
  d.has_new = a.k_new != nullptr && (d.tok0 + d.rows == cur.len);
  d.pool_rows = d.has_new ? d.rows - 1 : d.rows;
  d.row0 = -1;
  if (a.page_size % ROWS == 0) {   // chunks start at multiples of ROWS, so the chunk sits inside one page
    int room;
    d.row0 = pool_row_index(a, d.seat, d.tok0, room);
  }
  return d;
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

struct DecodePlan {
  long long N;       // chunks of all seats
  long long c0, c1;  // this CTA's chunk range
  int Ge;            // effective CTA count
  int H;             // > 0: pair-weighted split (see chunk_start), else uniform
  SeatCursor cur;    // positioned on the seat holding chunk c0
};

// Work split of CTAs that each run NS chunk streams (the dedicated-producer kernel): stream v of block x is split slot
// c = NS * x + v of G, the grid's stream count. decode_plan below is the one-stream form, kept separate so the
// register allocation of the one-stream kernels does not carry the per-stream state. Every thread of the CTA calls
// it, naming the stream it works for (mine); P receives that stream's plan. Returns the mask of streams that have
// chunks (bit v: stream v). Also writes zeros for seats with nothing to attend and flags lengths beyond the block table's
// capacity.
template <int ROWS, int WARPS, int NS>
__device__ __forceinline__ unsigned decode_plan_streams(const DecodeArgs& a, int G, int mine, DecodePlan& P) {
  constexpr int kThreads = WARPS * 32;
  __shared__ long long warp_sums[WARPS];
  __shared__ long long plan_first[NS];
  __shared__ int plan_seat[NS];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cbase = NS * static_cast<int>(blockIdx.x);
  const bool append = a.k_new != nullptr;

  long long local = 0;
  for (int s = tid; s < a.B; s += kThreads) {
    const int L = seat_tokens(a, s);
    local += (L + ROWS - 1) / ROWS;
    if (cbase == 0) {
      const int raw = a.seqlens[s] + (append ? 1 : 0);
      if (raw > a.max_pages * a.page_size || a.seqlens[s] < 0) atomicOr(a.status, kStatusBadLength);
    }
    const int owner = s % G;   // empty cache, nothing appended: the output is zero (as flash-attn writes)
    if (L == 0 && owner >= cbase && owner < cbase + NS) {
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
  for (int w = 0; w < WARPS; ++w) N += warp_sums[w];
  // Effective split count: never more streams than chunks, so every stream in [0, Ge) owns at least one chunk and the
  // streams between a seat's first and last owner all contribute a partial (the merge counts them).
  const int Ge = static_cast<int>(N < G ? N : G);
  // pair weighting only for the full two-per-SM grid of one-stream CTAs and enough chunks that every CTA keeps several
  const int H = (NS == 1 && a.pair_split > 0 && Ge == G && G == 2 * a.pair_split && N >= 4ll * Ge) ? a.pair_split : 0;
  const int nact = Ge - cbase < 0 ? 0 : (Ge - cbase > NS ? NS : Ge - cbase);   // streams 0 .. nact-1 have chunks
  if (nact == 0) return 0u;  // uniform across the CTA (the scan's first barrier orders the reads of warp_sums above)

  long long base = 0;
  for (int t0 = 0; t0 < a.B; t0 += kThreads) {
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
    for (int w = 0; w < WARPS; ++w) {
      if (w < warp) before += warp_sums[w];
      total += warp_sums[w];
    }
    incl += before;
    const long long excl = incl - n;
    for (int v = 0; v < nact; ++v) {
      const long long cv = chunk_start(cbase + v, N, Ge, H);
      if (n > 0 && base + excl <= cv && cv < base + incl) {
        plan_seat[v] = s;
        plan_first[v] = base + excl;
      }
    }
    base += total;
    __syncthreads();
    if (base > chunk_start(cbase + nact - 1, N, Ge, H)) break;   // uniform; the streams' first chunks ascend
  }
  __syncthreads();
  const bool act = mine < nact;
  P.N = N;
  P.Ge = Ge;
  P.H = H;
  P.c0 = act ? chunk_start(cbase + mine, N, Ge, H) : 0;
  P.c1 = act ? chunk_start(cbase + mine + 1, N, Ge, H) : 0;
  P.cur.seat = act ? plan_seat[mine] : 0;
  P.cur.first = act ? plan_first[mine] : 0;
  P.cur.len = act ? seat_tokens(a, plan_seat[mine]) : 0;
  P.cur.nch = (P.cur.len + ROWS - 1) / ROWS;
  return (1u << nact) - 1u;
}

// Work split of the CTA; every thread of the CTA calls it. Returns false when the CTA has no chunk. Also writes zeros
// for seats with nothing to attend and flags lengths beyond the block table's capacity.
template <int ROWS, int WARPS = kDecodeWarps>
__device__ __forceinline__ bool decode_plan(const DecodeArgs& a, DecodePlan& P) {
  constexpr int kThreads = WARPS * 32;
  __shared__ long long warp_sums[WARPS];
  __shared__ long long plan_first;
  __shared__ int plan_seat;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, c = blockIdx.x;   // G: launched CTAs (the split is re-derived from N)
  const bool append = a.k_new != nullptr;

  long long local = 0;
  for (int s = tid; s < a.B; s += kThreads) {
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
  for (int w = 0; w < WARPS; ++w) N += warp_sums[w];
  // Effective CTA count: never more CTAs than chunks, so every CTA in [0, Ge) owns at least one chunk and the CTAs
  // between a seat's first and last owner all contribute a partial (the merge counts them).
  const int Ge = static_cast<int>(N < G ? N : G);
  if (c >= Ge) return false;   // uniform across the CTA
  // pair weighting only for the full two-per-SM grid and enough chunks that every CTA keeps several
  const int H = (a.pair_split > 0 && Ge == G && G == 2 * a.pair_split && N >= 4ll * Ge) ? a.pair_split : 0;
  const long long c0 = chunk_start(c, N, Ge, H), c1 = chunk_start(c + 1, N, Ge, H);

  long long base = 0;
  for (int t0 = 0; t0 < a.B; t0 += kThreads) {
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
    for (int w = 0; w < WARPS; ++w) {
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
  __syncthreads();
  P.N = N;
  P.c0 = c0;
  P.c1 = c1;
  P.Ge = Ge;
  P.H = H;
  P.cur.seat = plan_seat;
  P.cur.first = plan_first;
  P.cur.len = seat_tokens(a, plan_seat);
  P.cur.nch = (P.cur.len + ROWS - 1) / ROWS;
  return true;
}

// Merge, in CTA order, the partials that CTAs c_first..c_last left for both q heads of (seat, KV head h), write the
// output rows and reset the seat's ticket counter for the next launch. Called by the warp that took the last ticket.
__device__ __forceinline__ void merge_seat_partials(const DecodeArgs& a, const SeatCursor& cur, int h, int lane,
                                                    int c_first, int c_last, __nv_bfloat16* op) {
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

// End of a seat's chunks in split slot c (the CTA, or one chunk stream of it) for KV head h. o0/o1 hold this lane's dims 4*lane..4*lane+3 of q heads 2h and
// 2h+1 (not yet divided by the sums); m0/m1 the running maxima (log2 domain), l0/l1 the running sums. A seat wholly
// inside this CTA is written directly; otherwise this CTA's partial goes to the workspace and the last CTA to arrive
// (atomic ticket) merges all partials of the seat in CTA order and writes the output.
__device__ __forceinline__ void decode_finish_seat(const DecodeArgs& a, const DecodePlan& P, int c,
                                                   const SeatCursor& cur, int h, int lane, float4 o0, float4 o1,
                                                   float m0, float m1, float l0, float l1) {
  const int c_first = cta_of_chunk(cur.first, P.N, P.Ge, P.H);
  const int c_last = cta_of_chunk(cur.first + cur.nch - 1, P.N, P.Ge, P.H);
  __nv_bfloat16* op = a.out + static_cast<long long>(cur.seat) * a.out_stride + (2 * h) * kHeadDim + 4 * lane;
  if (c_first == c_last) {
    const float r0 = 1.f / l0, r1 = 1.f / l1;
    *reinterpret_cast<uint2*>(op) = float4_to_bf16x4(make_float4(o0.x * r0, o0.y * r0, o0.z * r0, o0.w * r0));
    *reinterpret_cast<uint2*>(op + kHeadDim) = float4_to_bf16x4(make_float4(o1.x * r1, o1.y * r1, o1.z * r1, o1.w * r1));
    return;
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
  if (ticket != static_cast<unsigned>(c_last - c_first)) return;
  merge_seat_partials(a, cur, h, lane, c_first, c_last, op);
}

}  // namespace q3
