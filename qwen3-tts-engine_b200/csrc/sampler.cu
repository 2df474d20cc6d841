// Logit processing + top-k / temperature sampling, one CTA per row (sm_100a).
//
// Replaces, per sampled token of a frame:
//   Talker._cb0_logits (engine/talker.py:90-94): lg.float(); repetition penalty over the seat's `seen` row
//     (where(lg < 0, lg * rep, lg / rep)); + the suppress row; EOS masked to -inf while ngen[seat] < min_new
//   sample_topk (engine/ops.py:68-76): topk(k) -> softmax(vals / temperature) -> multinomial(1) -> gather
//   the embedding lookup of the sampled id that feeds the next step (engine/code_predictor.py:68, 71)
// k = 1 is greedy (the row's maximum; equal maxima resolve to the lowest index): one block-wide max over
// (key, -index), no selection.
//
// Selection (k > 1): the processed row is held as order-preserving 32-bit keys, 16 per thread at most (vocab <= 4096).
// The k-th largest key T is found by a 4-pass most-significant-digit radix select over 8-bit digits (a shared 256-bin
// histogram per pass); the k winners are the keys above T and the lowest-index keys equal to T. They are placed by
// shared-memory atomics (order is irrelevant: they are ranked next) -- the keys equal to T into a side list whose
// lowest indices are kept -- unless more than kSampleMaxTopK keys equal T (massive ties), in which case an ordered
// block scan gathers them. The winners are then ranked by (value desc, index asc).
// Sampling: p_j = exp((v_j - v_0) / T) over the sorted winners; one uniform u in [0, 1) from Philox4x32-10 (Salmon,
// Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011) keyed by the caller's seed with counter
// (row, launch index); the pick is the first j whose inclusive prefix sum exceeds u * sum. The launch index lives in
// device memory: every CTA reads it and then takes an atomic ticket, and the CTA holding the last ticket (every CTA
// has read the index by then) advances it, so CUDA-graph replays draw fresh numbers and a run is reproducible from
// (seed, starting index). The ticket is taken at the start, off the end of the kernel's critical path.
#include "q3_common.cuh"
#include "q3_kernels.h"

namespace q3 {

constexpr int kSampleThreads = 256;
constexpr int kSampleMaxVocab = 4096;
constexpr int kSamplePerThread = kSampleMaxVocab / kSampleThreads;   // 16

__device__ __forceinline__ uint32_t float_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Philox4x32 with 10 rounds (the published round function and constants).
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k.x += 0x9E3779B9u;
      k.y += 0xBB67AE85u;
    }
    const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
  }
  return c;
}

// Block-wide exclusive prefix count of `flag` in thread order, and the block total.
__device__ __forceinline__ int block_prefix_count(bool flag, int* warp_tot, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned m = __ballot_sync(0xffffffffu, flag);
  __syncthreads();   // warp_tot is reused across calls
  if (lane == 0) warp_tot[warp] = __popc(m);
  __syncthreads();
  int before = 0;
  total = 0;
#pragma unroll
  for (int w = 0; w < kSampleThreads / 32; ++w) {
    const int t = warp_tot[w];
    before += (w < warp) ? t : 0;
    total += t;
  }
  return before + __popc(m & ((1u << lane) - 1u));
}

__global__ void __launch_bounds__(kSampleThreads) sample_topk_kernel(const SampleArgs a) {
  __shared__ unsigned hist[256];
  __shared__ int warp_tot[kSampleThreads / 32];
  __shared__ uint32_t cand_key[kSampleMaxTopK];
  __shared__ int cand_idx[kSampleMaxTopK];
  __shared__ uint32_t sort_key[kSampleMaxTopK];
  __shared__ int sort_idx[kSampleMaxTopK];
  __shared__ int eq_idx[kSampleMaxTopK];
  __shared__ unsigned long long warp_best[kSampleThreads / 32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_krem;
  __shared__ unsigned s_eq;
  __shared__ int s_ngt, s_neq;
  __shared__ int s_pick;
  __shared__ unsigned long long s_launch;

  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const int V = a.V, K = a.k;
  if (tid == 0) {
    s_launch = *reinterpret_cast<volatile unsigned long long*>(a.rng_state);
    __threadfence();   // the read of the launch index is performed before this CTA's ticket
    const unsigned long long t = atomicAdd(a.rng_state + 1, 1ull);
    if (t == static_cast<unsigned long long>(gridDim.x) - 1) {   // the last ticket: reset it, advance the index
      a.rng_state[1] = 0ull;
      atomicAdd(a.rng_state, 1ull);
    }
  }
  if (tid < kSampleMaxTopK) {   // defined contents whatever the selection leaves: every index read below is < V
    cand_key[tid] = 0u;
    cand_idx[tid] = 0;
    sort_key[tid] = 0u;
    sort_idx[tid] = 0;
  }

  // ---- processed row -> keys (engine/talker.py:91-94 order: penalty, + bias, EOS mask)
  long long seat = 0;
  bool eos_masked = false;
  const uint8_t* seen_row = nullptr;
  if (a.seat) seat = a.seat[b];
  if (a.seen) seen_row = a.seen + seat * a.seen_stride;
  if (a.ngen) eos_masked = a.ngen[seat] < a.min_new;
  uint32_t key[kSamplePerThread];
#pragma unroll
  for (int j = 0; j < kSamplePerThread; ++j) {
    const int v = j * kSampleThreads + tid;
    key[j] = 0u;   // below every float key: never selected
    if (v < V) {
      float x = a.logits_bf16
                    ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.logits)[b * a.row_stride + v])
                    : reinterpret_cast<const float*>(a.logits)[b * a.row_stride + v];
      if (seen_row && seen_row[v]) x = x < 0.f ? x * a.rep : x / a.rep;
      if (a.bias) x = x + a.bias[v];
      if (eos_masked && v == a.eos) x = -INFINITY;
      key[j] = float_key(x);
    }
  }

  if (K == 1) {
    // ---- greedy: the largest (key, -index); padding slots never compete
    unsigned long long best = 0ull;
#pragma unroll
    for (int j = 0; j < kSamplePerThread; ++j) {
      const int v = j * kSampleThreads + tid;
      if (v < V) {
        const unsigned long long c = (static_cast<unsigned long long>(key[j]) << 32) | (0xffffffffu - static_cast<uint32_t>(v));
        best = c > best ? c : best;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, best, o);
      best = y > best ? y : best;
    }
    if (lane == 0) warp_best[tid >> 5] = best;
    __syncthreads();
    if (tid == 0) {
      unsigned long long m = warp_best[0];
#pragma unroll
      for (int w = 1; w < kSampleThreads / 32; ++w) m = warp_best[w] > m ? warp_best[w] : m;
      const int id = static_cast<int>(0xffffffffu - static_cast<uint32_t>(m));
      s_pick = id;
      a.out_ids[b * a.out_stride] = id;
    }
    __syncthreads();
  } else {
  // ---- radix select of the K-th largest key
  if (tid == 0) {
    s_prefix = 0u;
    s_krem = K;
    s_eq = 0u;
    s_ngt = 0;
    s_neq = 0;
  }
  uint32_t mask = 0u;
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    hist[tid] = 0u;
    __syncthreads();
    const uint32_t prefix = s_prefix;
#pragma unroll
    for (int j = 0; j < kSamplePerThread; ++j) {
      const int v = j * kSampleThreads + tid;
      if (v < V && (key[j] & mask) == prefix) atomicAdd(&hist[(key[j] >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid < 32) {
      // lane l owns digits 255-8l .. 248-8l (descending); find the digit where the count from the top reaches krem
      unsigned c[8], s = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        c[i] = hist[255 - 8 * lane - i];
        s += c[i];
      }
      unsigned incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const unsigned excl = incl - s;
      const int krem = s_krem;
      const unsigned hit = __ballot_sync(0xffffffffu, incl >= static_cast<unsigned>(krem));
      const int first = __ffs(hit) - 1;   // krem <= elements matching the prefix, so some lane is hit
      if (lane == first) {
        unsigned above = excl, at = 0u;
        int d = 255 - 8 * lane;
        bool found = false;
#pragma unroll
        for (int i = 0; i < 8; ++i) {   // static indexing: c stays in registers
          if (!found && above + c[i] >= static_cast<unsigned>(krem)) {
            d = 255 - 8 * lane - i;
            at = c[i];
            found = true;
          }
          if (!found) above += c[i];
        }
        s_prefix = prefix | (static_cast<uint32_t>(d) << shift);
        s_krem = krem - static_cast<int>(above);
        s_eq = at;   // keys matching the new prefix (after the last pass: the keys equal to T)
      }
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t T = s_prefix;   // the K-th largest key; s_krem of the keys equal to it are taken
  const int take_eq = s_krem;
  const int eq_total = static_cast<int>(s_eq);

  if (eq_total <= kSampleMaxTopK) {
    // ---- winners by atomics: keys > T (fewer than K of them) straight into cand, keys == T into eq_idx
#pragma unroll
    for (int j = 0; j < kSamplePerThread; ++j) {
      const int v = j * kSampleThreads + tid;
      if (v < V) {
        if (key[j] > T) {
          const int slot = atomicAdd(&s_ngt, 1);
          cand_key[slot] = key[j];
          cand_idx[slot] = v;
        } else if (key[j] == T) {
          eq_idx[atomicAdd(&s_neq, 1)] = v;
        }
      }
    }
    __syncthreads();
    if (tid < eq_total) {   // the take_eq lowest indices among the keys equal to T follow the keys above it
      const int mi = eq_idx[tid];
      int r = 0;
      for (int j = 0; j < eq_total; ++j) r += eq_idx[j] < mi ? 1 : 0;
      if (r < take_eq) {
        cand_key[s_ngt + r] = T;
        cand_idx[s_ngt + r] = mi;
      }
    }
  } else {
  // ---- gather the K winners in index order (keys > T, then the lowest-index keys == T)
  int gt_run = 0, eq_run = 0;
#pragma unroll
  for (int j = 0; j < kSamplePerThread; ++j) {
    if (j * kSampleThreads >= V) continue;   // uniform across the CTA (the scans below synchronise it)
    const int v = j * kSampleThreads + tid;
    const bool gt = v < V && key[j] > T;
    const bool eq = v < V && key[j] == T;
    int gt_tot, eq_tot;
    const int gt_before = block_prefix_count(gt, warp_tot, gt_tot);
    const int eq_before = block_prefix_count(eq, warp_tot, eq_tot);
    const int eb = eq_run + eq_before;
    if (gt || (eq && eb < take_eq)) {
      const int slot = gt_run + gt_before + min(eb, take_eq);
      if (slot < kSampleMaxTopK) {
        cand_key[slot] = key[j];
        cand_idx[slot] = v;
      }
    }
    gt_run += gt_tot;
    eq_run += eq_tot;
  }
  }
  __syncthreads();

  // ---- rank the winners by (value desc, index asc)
  if (tid < K) {
    const uint32_t mk = cand_key[tid];
    const int mi = cand_idx[tid];
    int r = 0;
    for (int j = 0; j < K; ++j) {
      const uint32_t ok = cand_key[j];
      r += (ok > mk || (ok == mk && cand_idx[j] < mi)) ? 1 : 0;
    }
    sort_key[r] = mk;
    sort_idx[r] = mi;
  }
  __syncthreads();

  // ---- temperature softmax over the sorted winners and one multinomial draw
  if (tid < 32) {
    int pick = 0;
    if (K > 1) {
      const float v0 = key_float(sort_key[0]);
      const float it = a.inv_temp;
      const float va = lane < K ? key_float(sort_key[lane]) : -INFINITY;
      const float vb = lane + 32 < K ? key_float(sort_key[lane + 32]) : -INFINITY;
      float ea = (lane < K && v0 > -INFINITY) ? expf((va - v0) * it) : 0.f;
      float eb = (lane + 32 < K && v0 > -INFINITY) ? expf((vb - v0) * it) : 0.f;
      float ca = ea, cb = eb;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float ya = __shfl_up_sync(0xffffffffu, ca, o);
        const float yb = __shfl_up_sync(0xffffffffu, cb, o);
        if (lane >= o) {
          ca += ya;
          cb += yb;
        }
      }
      const float tot_a = __shfl_sync(0xffffffffu, ca, 31);
      cb += tot_a;
      const float total = __shfl_sync(0xffffffffu, cb, 31);
      const uint4 r = philox4x32_10(
          make_uint4(static_cast<uint32_t>(b), static_cast<uint32_t>(s_launch), static_cast<uint32_t>(s_launch >> 32),
                     0u),
          make_uint2(static_cast<uint32_t>(a.seed), static_cast<uint32_t>(a.seed >> 32)));
      const float u = static_cast<float>(r.x >> 8) * (1.f / 16777216.f);
      const float target = u * total;
      const unsigned ha = __ballot_sync(0xffffffffu, lane < K && ea > 0.f && ca > target);
      const unsigned hb = __ballot_sync(0xffffffffu, lane + 32 < K && eb > 0.f && cb > target);
      if (ha) {
        pick = __ffs(ha) - 1;
      } else if (hb) {
        pick = 32 + __ffs(hb) - 1;
      } else {   // u * total rounded onto the total: the last winner with any weight
        const unsigned la = __ballot_sync(0xffffffffu, lane < K && ea > 0.f);
        const unsigned lb = __ballot_sync(0xffffffffu, lane + 32 < K && eb > 0.f);
        pick = lb ? 32 + 31 - __clz(lb) : (la ? 31 - __clz(la) : 0);
      }
    }
    if (lane == 0) {
      s_pick = sort_idx[pick];
      a.out_ids[b * a.out_stride] = sort_idx[pick];
    }
  }
  __syncthreads();
  }

  // ---- the embedding row of the sampled id
  if (a.emb) {
    const long long id = s_pick;
    const uint2* src = reinterpret_cast<const uint2*>(a.emb + id * a.emb_stride);
    uint2* dst = reinterpret_cast<uint2*>(a.emb_out + b * a.emb_out_stride);
    for (int i = tid; i < a.emb_dim / 4; i += kSampleThreads) dst[i] = src[i];
  }
}

cudaError_t launch_sample_topk(const SampleArgs& a, cudaStream_t stream) {
  if (a.B == 0) return cudaSuccess;
  sample_topk_kernel<<<a.B, kSampleThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace q3
