// Prompt prefill attention, warp-specialised and TMA-fed, on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Same contract as prefill_kernel (prefill.cu): replaces flash_attn_varlen_func (engine/talker.py:169) and
// flash_attn_func over a cached prefix (engine/arrivals.py:148); sequence i has R_i query rows, N_i new key rows and
// P_i cached prefix keys in its pages, keys indexed prefix first, causal aligned to the bottom right.
//
// One CTA = (64-position query tile, KV head h, sequence); its 128 accumulator rows are the 64 positions of q heads 2h
// and 2h+1, which share every K/V tile. Six warps with fixed roles:
//   warp 4 (producer)   lane 0 issues TMA tensor copies (cp.async.bulk.tensor, no multicast, this GPU's memory only):
//                       the Q tile once, then K and V tiles of 64 keys into two 2-slot rings, 128-byte swizzled so they
//                       are UMMA operands as they land; K(t+2) goes out as soon as S(t) has read K(t), V(t+2) once
//                       P(t) V(t) is done. Prefix keys come page by page out of the pool, new keys as one box per 64
//                       rows. With write_kv it also stores the new K/V tiles this CTA owns into the pages (TMA tensor
//                       stores from the same shared-memory tiles, page-aligned boxes).
//   warp 5 (MMA)        lane 0 issues S(t) = Q K(t)^T into one of two TMEM S buffers once K(t) has landed and
//                       P(t-2) V(t-2) (whose P sat in that buffer) is done; tcgen05.commit arrives on the K-slot-free
//                       and S-ready barriers.
//   warps 0-3 (softmax) thread r owns TMEM lane r = accumulator row r: reads S(t) (tcgen05.ld), online softmax in the
//                       exp2 domain with a lazy running max (O rescaled in TMEM only when a max grows by more than 2^8),
//                       writes P(t) as bf16 into TMEM over S(t) (tcgen05.st); lane 0 of warp 0 then issues O += P(t)
//                       V(t) into the TMEM O accumulator itself (A from TMEM, V from shared memory) as soon as all four
//                       warps have written P(t), committing to the V-slot-free and P.V-done barriers. At the end the
//                       warps divide O by the row sums and store the output rows. Page-write rows that do not fill a page-aligned box
//                       (a prefix not aligned to the box, a last partial box) are copied by these threads at the start.
// While the softmax warps work on S(t), the tensor core computes S(t+1) and P(t-1) V(t-1), and the producer loads the
// next tiles. Shared memory: Q 32 KB + K 2 x 16 KB + V 2 x 16 KB = 96 KB (+ alignment slack); TMEM 256 columns (S0,
// S1, O; P(t) is written as bf16 over S(t) once S(t) is read, and the P.V MMA takes its A operand from there): two CTAs
// per SM. Every mbarrier wait is bounded (2 s); a timed-out role raises the status bit and an abort flag the other
// roles poll, in-flight copies and MMAs are waited for (bounded), and TMEM is always freed.
#include <cuda.h>

#include <cstring>

#include "prefill_common.cuh"
#include "tensor_map.cuh"

namespace q3 {

namespace {

constexpr int kTwProducerWarp = 4, kTwMmaWarp = 5;
constexpr int kTwThreads = 6 * 32;
constexpr int kTwTmemCols = 256;
constexpr uint32_t kTwOCol = 128;             // S(t) at column 64 * (t & 1), O at 128

struct TwSmem {
  static constexpr int kQ = 0;                // [2 dim halves][128 rows][128 B]: 32 KB, SW128 K-major
  static constexpr int kK = 32768;            // K slot s at kK + s * kTile: [2 dim halves][64 keys][128 B]
  static constexpr int kV = 65536;            // V slot s at kV + s * kTile: same layout (MN-major B operand)
  static constexpr int kTile = 16384;
  static constexpr int kHalf = 8192;          // one dim half of a K or V tile
  static constexpr int kBars = 98304;
  // Barriers, every one waited with a parity that is never ambiguous: a waiter is at most one phase away from its
  // barrier's next completion (each role waits for every phase of the barriers it waits on, in order, and no role can
  // complete a barrier twice before its waiter has seen the first completion).
  static constexpr int kQFull = 0, kKFull = 1, kVFull = 3, kKEmpty = 5, kVEmpty = 7, kSFull = 9, kPFull = 11,
                       kPvDone = 13, kFinal = 15, kFinalPv = 16;
  static constexpr int kNumBars = 17;
  static constexpr int kTmemSlot = kBars + 8 * kNumBars;
  static constexpr int kAbort = kTmemSlot + 4;
  static constexpr int kIssuedK = kAbort + 4;  // K and V tiles the producer has issued (read on the abort path)
  static constexpr int kIssuedV = kIssuedK + 4;
  static constexpr int kBytes = kIssuedV + 4;
  static constexpr int kAlloc = kBytes + 1024;   // + slack to align the base to 1024 B (128-byte swizzle atoms)
};

struct PfTmaParams {
  PrefillArgs a;
  CUtensorMap tq;    // q rows    [q_rows][16 heads][128]
  CUtensorMap tk;    // new keys  [kv_rows][8 heads][128]
  CUtensorMap tv;
  CUtensorMap tkp;   // pools     [num_pages * page_size][8 heads][128] (prefix reads, page-write stores)
  CUtensorMap tvp;
  CUtensorMap to;    // output rows [q_rows][16 heads][128]
  int box_rows;      // rows per pool box: min(page_size, 64)
  int pool_maps;     // tkp / tvp are valid
};

// UMMA shared-memory descriptor of a 128-byte-swizzled operand: 8-row groups `sbo` bytes apart; `lbo` = the distance
// between 64-element column blocks for an MN-major operand (unused, 16, for K-major).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t sbo, uint32_t lbo) {
  uint64_t d = static_cast<uint64_t>((addr >> 4) & 0x3fff);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3fff) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3fff) << 32;
  d |= static_cast<uint64_t>(1) << 46;        // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;        // layout: 128-byte swizzle
  return d;
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Shared -> global tensor store (a page-aligned box of new K or V rows into the pool), in this thread's bulk group.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// This thread's bulk stores have finished reading shared memory (the slot may be refilled).
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Number of new-key tiles the query tile q of a sequence visits (the key tiles past the prefix).
__device__ __forceinline__ int new_tiles_of(const PfSeq& s, int q, int causal) {
  const int L = s.P + s.Nn, shift = L - s.R;
  const int key_end = causal ? min(L, shift + min(s.R - 1, q * 64 + 63) + 1) : L;
  return (max(key_end - s.P, 0) + 63) / 64;
}

// Wait for phase `parity` of `bar`; false after 2 s or once another role has raised the abort flag.
__device__ __forceinline__ bool tw_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
#pragma unroll 1
  for (int i = 0; i < 1024; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
#pragma unroll 1
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > 2000000000ull) return false;
  }
}

__device__ __forceinline__ void tw_fail(uint32_t* status, volatile int* abort_flag) {
  atomicOr(status, kStatusWaitTimeout);
  *abort_flag = 1;
}

// The page writes of a chunked prefill (write_kv) for KV head h: new rows [r0, r1) of the sequence go to positions
// P + r of its seat's pages, K and V (256 bytes each per row and head), by 128 threads with 16-byte accesses, eight loads
// in flight before their stores. The attention reads new keys from the input rows and only the prefix from the pages,
// so these writes never race with its reads of valid keys.
__device__ __forceinline__ void write_new_rows(const PrefillArgs& a, const PfSeq& s, int h, int r0, int r1, int tid) {
  const int n = (r1 - r0) * 32;                               // 16-byte pieces: 16 per row for K and 16 for V
#pragma unroll 1
  for (int base = 0; base < n; base += 8 * 128) {
    uint4 v[8];
    uint4* dst[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * 128 + tid;
      dst[u] = nullptr;
      if (i < n) {
        const int r = r0 + (i >> 5), which = (i >> 4) & 1, c = i & 15;
        const __nv_bfloat16* src = (which ? a.v : a.k) + static_cast<long long>(s.k0 + r) * a.kv_stride + h * kHeadDim;
        v[u] = __ldg(reinterpret_cast<const uint4*>(src) + c);
        __nv_bfloat16* pool = which ? a.v_pool : a.k_pool;
        dst[u] = reinterpret_cast<uint4*>(pool + pf_pool_row(a, s.seat, s.P + r) * (kKvHeads * kHeadDim) +
                                          h * kHeadDim) + c;
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (dst[u] != nullptr) *dst[u] = v[u];
  }
}

__global__ void __launch_bounds__(kTwThreads, 2) prefill_tma_kernel(const __grid_constant__ PfTmaParams p) {
  const PrefillArgs& a = p.a;
  extern __shared__ __align__(1024) uint8_t tw_raw[];
  uint8_t* smem = tw_raw + ((1024u - (smem_addr(tw_raw) & 1023u)) & 1023u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == kTwProducerWarp * 32) {   // the descriptors travel while the sequence geometry loads
    prefetch_map(&p.tq);
    prefetch_map(&p.tk);
    prefetch_map(&p.tv);
    prefetch_map(&p.to);
  }
  // grid (sequence, KV head, query tile from the last): blocks launch in linear order, so every sequence's heaviest
  // (latest) query tile goes out in the first wave and the light ones fill the tail
  const int h = blockIdx.y;
  const PfSeq s = pf_seq(a, blockIdx.x);
  if (s.R <= 0) {                                             // no queries: CTA 0 still writes the new rows (write_kv)
    if (a.write_kv && blockIdx.z == 0 && tid < 128) write_new_rows(a, s, h, 0, s.Nn, tid);
    return;
  }
  const int ntq = (s.R + 63) / 64;
  const int qt = ntq - 1 - static_cast<int>(blockIdx.z);
  if (qt < 0) return;                                         // uniform per CTA; nothing allocated yet

  // ---- key tiles: the prefix keys [0, P) in tiles of 64, then the new keys [0, N) in tiles of 64 (combined index
  //      P + j), each tile from one source; only the keys some row of this query tile can see are visited
  const int L = s.P + s.Nn, shift = L - s.R;
  const int last_row = min(s.R - 1, qt * 64 + 63);
  const int key_end = a.causal ? min(L, shift + last_row + 1) : L;
  const int n_pre = (min(key_end, s.P) + 63) / 64;
  const int n_new = (max(key_end - s.P, 0) + 63) / 64;
  const int ntk = n_pre + n_new;                              // >= 1: key 0 is visible to every row

  // ---- page writes (write_kv): this CTA owns new-key tiles [u_lo, n_new), the ones the previous query tile does not
  //      visit (a partition of all new tiles over the query tiles). Rows in whole page-aligned boxes go out by TMA
  //      stores from the loaded tiles; the rest (misaligned prefix, last partial box) by the softmax threads.
  const int u_lo = qt > 0 ? new_tiles_of(s, qt - 1, a.causal) : 0;
  const bool tma_store = a.write_kv && p.pool_maps && (s.P % p.box_rows) == 0;
  const int box_end = tma_store ? (s.Nn / p.box_rows) * p.box_rows : 64 * u_lo;   // rows [64 u_lo, box_end): TMA
  const int own_end = min(s.Nn, 64 * n_new);                                        // rows [64 u_lo, own_end) owned

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TwSmem::kBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TwSmem::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + TwSmem::kAbort);
  volatile int* issued_k = reinterpret_cast<volatile int*>(smem + TwSmem::kIssuedK);
  volatile int* issued_v = reinterpret_cast<volatile int*>(smem + TwSmem::kIssuedV);
  const uint32_t sbase = smem_addr(smem);

  if (warp == kTwMmaWarp) {   // TMEM: 256 columns; shared memory limits an SM to two CTAs, so 512 columns suffice
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTwTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == kTwProducerWarp * 32) {
    mbar_init(&bars[TwSmem::kQFull], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[TwSmem::kKFull + i], 1);
      mbar_init(&bars[TwSmem::kVFull + i], 1);
      mbar_init(&bars[TwSmem::kKEmpty + i], 1);
      mbar_init(&bars[TwSmem::kVEmpty + i], 1);
      mbar_init(&bars[TwSmem::kSFull + i], 1);
      mbar_init(&bars[TwSmem::kPFull + i], 4);               // one arrival per softmax warp
      mbar_init(&bars[TwSmem::kPvDone + i], 1);
    }
    mbar_init(&bars[TwSmem::kFinal], 1);
    mbar_init(&bars[TwSmem::kFinalPv], 1);
    *abort_flag = 0;
    *issued_k = 0;
    *issued_v = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTwProducerWarp) {
    // ------------------------------------------------------------------ producer: TMA copies and page stores
    if (lane == 0) {
      const uint32_t qbar = smem_addr(&bars[TwSmem::kQFull]);
      mbar_arrive_expect_tx(&bars[TwSmem::kQFull], 32768u);
      for (int g = 0; g < 2; ++g)
        for (int half = 0; half < 2; ++half)
          tma_load_3d(sbase + TwSmem::kQ + half * 16384 + g * 8192, &p.tq, half * 64, 2 * h + g, s.q0 + qt * 64, qbar);
      // one K or V tile of key tile t into slot t & 1
      auto load_tile = [&](int t, bool is_v) {
        const int st = t & 1;
        uint64_t* fb = &bars[(is_v ? TwSmem::kVFull : TwSmem::kKFull) + st];
        const uint32_t fbar = smem_addr(fb);
        const uint32_t dst = sbase + (is_v ? TwSmem::kV : TwSmem::kK) + st * TwSmem::kTile;
        mbar_arrive_expect_tx(fb, static_cast<uint32_t>(TwSmem::kTile));
        if (t < n_pre) {
          const CUtensorMap* m = is_v ? &p.tvp : &p.tkp;
          for (int r0 = 0; r0 < 64; r0 += p.box_rows) {
            const int tok = t * 64 + r0;
            // rows past the prefix in its last tile: any valid pool row (their V rows are zeroed before P.V)
            const int row = tok < s.P ? static_cast<int>(pf_pool_row(a, s.seat, tok)) : 0;
            for (int half = 0; half < 2; ++half) tma_load_3d(dst + half * TwSmem::kHalf + r0 * 128, m, half * 64, h, row, fbar);
          }
        } else {
          const int row = s.k0 + (t - n_pre) * 64;            // rows past the tensor are zero-filled by the copy
          const CUtensorMap* m = is_v ? &p.tv : &p.tk;
          for (int half = 0; half < 2; ++half) tma_load_3d(dst + half * TwSmem::kHalf, m, half * 64, h, row, fbar);
        }
      };
      // the page stores of key tile t (a new-key tile this CTA owns), from slot t & 1: whole boxes below box_end
      auto store_tile = [&](int t, bool is_v) {
        const int u = t - n_pre;
        if (!tma_store || u < u_lo) return;
        const uint32_t src = sbase + (is_v ? TwSmem::kV : TwSmem::kK) + (t & 1) * TwSmem::kTile;
        const CUtensorMap* m = is_v ? &p.tvp : &p.tkp;
        for (int r0 = 0; r0 < 64 && 64 * u + r0 + p.box_rows <= box_end; r0 += p.box_rows) {
          const int row = static_cast<int>(pf_pool_row(a, s.seat, s.P + 64 * u + r0));
          for (int half = 0; half < 2; ++half) tma_store_3d(m, src + half * TwSmem::kHalf + r0 * 128, half * 64, h, row);
        }
        bulk_commit();
      };
      bool ok = true;
      for (int t = 0; t < ntk && ok; ++t) {
        for (int is_v = 0; is_v < 2; ++is_v) {
          if (t >= 2) {
            // the slot's previous tile (t - 2): its MMA reads are done; store it to the pages if this CTA owns it,
            // and let the stores finish reading before the slot is refilled
            const int e = (is_v ? TwSmem::kVEmpty : TwSmem::kKEmpty) + (t & 1);
            if (!tw_wait(&bars[e], ((t >> 1) - 1) & 1, abort_flag)) {
              tw_fail(a.status, abort_flag);
              ok = false;
              break;
            }
            store_tile(t - 2, is_v != 0);
            bulk_wait_read();
          }
          load_tile(t, is_v != 0);
          if (is_v) *issued_v = t + 1; else *issued_k = t + 1;
        }
      }
      // the last two tiles' page stores, once their data has landed
      if (ok && tma_store)
        for (int t = max(ntk - 2, n_pre + u_lo); t < ntk; ++t)
          for (int is_v = 0; is_v < 2; ++is_v) {
            const int f = (is_v ? TwSmem::kVFull : TwSmem::kKFull) + (t & 1);
            if (!tw_wait(&bars[f], (t >> 1) & 1, abort_flag)) {
              tw_fail(a.status, abort_flag);
              break;
            }
            store_tile(t, is_v != 0);
          }
      bulk_wait_read();   // the page stores have read shared memory (their global writes complete on their own)
    }
    __syncwarp();
  } else if (warp == kTwMmaWarp) {
    // ------------------------------------------------------------------ MMA issue: S(t) = Q K(t)^T, in order
    // S(t) goes into TMEM buffer t & 1 once K(t) has landed and P(t - 2) V(t - 2) is done (P(t - 2) was written over
    // S(t - 2) in that buffer). P V is issued by softmax warp 0 the moment P is written: no hand-over through this
    // warp. Every wait's outcome is agreed across the warp (__all_sync), so the lanes leave together.
    constexpr uint32_t kIdescQK = umma_idesc_bf16(128, 64, 0, 0);
    bool ok = __all_sync(0xffffffffu, tw_wait(&bars[TwSmem::kQFull], 0, abort_flag));
    for (int t = 0; ok && t < ntk; ++t) {
      ok = __all_sync(0xffffffffu, tw_wait(&bars[TwSmem::kKFull + (t & 1)], (t >> 1) & 1, abort_flag));
      if (ok && t >= 2)
        ok = __all_sync(0xffffffffu, tw_wait(&bars[TwSmem::kPvDone + (t & 1)], ((t - 2) >> 1) & 1, abort_flag));
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t sq = sbase + TwSmem::kQ, sk = sbase + TwSmem::kK + (t & 1) * TwSmem::kTile;
        const uint32_t t_s = tmem + 64u * static_cast<uint32_t>(t & 1);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_bf16(t_s, sw128_desc(sq + (ks >> 2) * 16384 + (ks & 3) * 32, 1024, 16),
                    sw128_desc(sk + (ks >> 2) * TwSmem::kHalf + (ks & 3) * 32, 1024, 16), kIdescQK, ks > 0 ? 1u : 0u);
        umma_commit(&bars[TwSmem::kKEmpty + (t & 1)]);
        umma_commit(&bars[TwSmem::kSFull + (t & 1)]);
      }
      __syncwarp();
    }
    if (!ok && lane == 0) tw_fail(a.status, abort_flag);
  } else {
    // ------------------------------------------------------------------ softmax + epilogue (warps 0-3)
    const int row = tid;                                       // TMEM lane = accumulator row
    const int row_g = row >> 6, row_j = qt * 64 + (row & 63);
    const bool row_valid = row_j < s.R;
    const int my_limit = (a.causal && row_valid) ? shift + row_j : L - 1;   // last visible key of this row
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    if (a.write_kv && max(box_end, 64 * u_lo) < own_end)      // owned rows no TMA store covers
      write_new_rows(a, s, h, max(box_end, 64 * u_lo), own_end, tid);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int t = 0; t < ntk; ++t) {
      const int b = t & 1;
      ok = tw_wait(&bars[TwSmem::kSFull + b], (t >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) tw_fail(a.status, abort_flag);
        break;
      }
      tc_fence_after();
      float sv[2][32];
      tmem_ld32(tmem + 64u * b + lane_base, sv[0]);
      tmem_ld32(tmem + 64u * b + 32u + lane_base, sv[1]);
      tc_wait_ld();
      int kbase, kcount;
      if (t < n_pre) {
        kbase = t * 64;
        kcount = min(64, s.P - kbase);
      } else {
        const int u = t - n_pre;
        kbase = s.P + u * 64;
        kcount = min(64, s.Nn - u * 64);
      }
      const int vis_n = min(kcount, my_limit - kbase + 1);     // keys [0, vis_n) of this tile are visible
      // raw maxima (the scale is positive, so it is applied once to the maximum), masked keys set to -inf
      float cm4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (__all_sync(0xffffffffu, vis_n >= 64)) {
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int i = 0; i < 32; ++i) cm4[i & 3] = fmaxf(cm4[i & 3], sv[u][i]);
      } else {
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            sv[u][i] = (u * 32 + i < vis_n) ? sv[u][i] : -INFINITY;
            cm4[i & 3] = fmaxf(cm4[i & 3], sv[u][i]);
          }
      }
      const float cmax = fmaxf(fmaxf(cm4[0], cm4[1]), fmaxf(cm4[2], cm4[3])) * a.scale_log2;
      // the running max moves (and O is rescaled) only when it would grow by more than 8 (a factor 256 in P)
      const bool grow = cmax > m_run + 8.f || (m_run == -INFINITY && cmax > -INFINITY);
      const float m_new = grow ? cmax : m_run;
      const float alpha = grow ? exp2f(m_run - m_new) : 1.f;  // 0 on the first visible tile
      const float mm = m_new == -INFINITY ? 0.f : m_new;
      // p = 2^(s * scale - m) by packed FMAs into the approximate exp2; row sums by packed adds in 4 chains
      const float2 sc2 = make_float2(a.scale_log2, a.scale_log2), nm2 = make_float2(-mm, -mm);
      float2 ls2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      uint32_t pk[32];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 x = __ffma2_rn(make_float2(sv[u][i], sv[u][i + 1]), sc2, nm2);
          const float2 pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
          ls2[(i >> 1) & 3] = __fadd2_rn(ls2[(i >> 1) & 3], pp);
          pk[u * 16 + i / 2] = pack_bf16x2(pp.x, pp.y);
        }
      const float2 lsa = __fadd2_rn(__fadd2_rn(ls2[0], ls2[1]), __fadd2_rn(ls2[2], ls2[3]));
      l_run = l_run * alpha + (lsa.x + lsa.y);
      m_run = m_new;
      if (t > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // rescale O where a max moved (tile 0 starts O from zero): O must hold P(t-1) V(t-1) first. Its barrier last
        // completed for P.V(t-3), which finished before S(t) was issued (S(t) waits for P.V(t-2)).
        ok = tw_wait(&bars[TwSmem::kPvDone + ((t - 1) & 1)], ((t - 1) >> 1) & 1, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
          if (lane == 0) tw_fail(a.status, abort_flag);
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tmem_ld32(tmem + kTwOCol + lane_base + c * 32, ov);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= alpha;
          tmem_st32(tmem + kTwOCol + lane_base + c * 32, ov);
        }
        tc_wait_st();
      }
      // ---- P(t) as bf16 into TMEM over S(t) (already read): lane r = row r, keys 2i and 2i+1 in column 64b + i, the
      //      layout the P.V MMA reads its A operand in
      tmem_st32u(tmem + 64u * b + lane_base, pk);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[TwSmem::kPFull + b]);
      if (warp == 0) {
        // ---- O += P(t) V(t), issued here once all four warps have written P(t) and V(t) has landed
        ok = __all_sync(0xffffffffu, tw_wait(&bars[TwSmem::kPFull + b], (t >> 1) & 1, abort_flag) &&
                                         tw_wait(&bars[TwSmem::kVFull + b], (t >> 1) & 1, abort_flag));
        if (!ok) {
          if (lane == 0) tw_fail(a.status, abort_flag);
          break;
        }
        // a tile's V rows past the end of its source (the prefix's last tile: stale page contents; the new keys'
        // last tile: rows of another sequence or of none) may hold anything, non-finite included: zero them, whole
        // 128-byte rows, so P = 0 meets V = 0 there
        const int first = t < n_pre ? s.P - t * 64 : s.Nn - (t - n_pre) * 64;
        if (first < 64) {
          uint8_t* vt = smem + TwSmem::kV + b * TwSmem::kTile;
          for (int i = lane; i < (64 - first) * 16; i += 32) {
            const int r = first + (i >> 4), half = (i >> 3) & 1, c = i & 7;
            *reinterpret_cast<uint4*>(vt + half * TwSmem::kHalf + r * 128 + c * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        tc_fence_after();
        if (lane == 0) {
          constexpr uint32_t kIdescPV = umma_idesc_bf16(128, kHeadDim, 0, 1);
          const uint32_t svv = sbase + TwSmem::kV + b * TwSmem::kTile;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_bf16_tmem_a(tmem + kTwOCol, tmem + 64u * b + 8u * ks, sw128_desc(svv + ks * 2048, 1024, TwSmem::kHalf),
                             kIdescPV, (t > 0 || ks > 0) ? 1u : 0u);
          umma_commit(&bars[TwSmem::kVEmpty + b]);
          umma_commit(&bars[TwSmem::kPvDone + b]);
        }
        __syncwarp();
      }
    }
    // ---- epilogue: O / l -> bf16 rows (every thread takes part in the warp-collective TMEM loads)
    if (ok) {
      ok = tw_wait(&bars[TwSmem::kPvDone + ((ntk - 1) & 1)], ((ntk - 1) >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0) tw_fail(a.status, abort_flag);
    }
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    if (ok) tc_fence_after();
    if (qt * 64 + 64 <= s.R) {
      // a full query tile: the rows go through shared memory (the Q buffer: the last S has read it) in the layout the
      // Q tile came in, and out as four TMA tensor stores (2 heads x 2 dim halves) issued by one thread. The named
      // barrier is reached by all four softmax warps on every path (ok is agreed per warp, not across warps).
      if (ok) {
        uint8_t* orow = smem + TwSmem::kQ + row_g * 8192 + (row & 63) * 128;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tmem_ld32(tmem + kTwOCol + lane_base + c * 32, ov);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            const int chunk = (c * 32 + i) >> 3;              // 16-byte chunk 0..15 of the 256-byte row
            uint4 w;
            w.x = pack_bf16x2(ov[i] * inv, ov[i + 1] * inv);
            w.y = pack_bf16x2(ov[i + 2] * inv, ov[i + 3] * inv);
            w.z = pack_bf16x2(ov[i + 4] * inv, ov[i + 5] * inv);
            w.w = pack_bf16x2(ov[i + 6] * inv, ov[i + 7] * inv);
            *reinterpret_cast<uint4*>(orow + (chunk >> 3) * 16384 + (((chunk & 7) ^ (row & 7)) << 4)) = w;
          }
        }
        fence_proxy_async_smem();
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");            // the four softmax warps only
      if (tid == 0 && !*abort_flag) {
        for (int g = 0; g < 2; ++g)
          for (int half = 0; half < 2; ++half)
            tma_store_3d(&p.to, sbase + TwSmem::kQ + half * 16384 + g * 8192, half * 64, 2 * h + g, s.q0 + qt * 64);
        bulk_commit();
        bulk_wait_read();                                     // shared memory stays valid until the stores read it
      }
    } else if (ok) {
      // the sequence's last, partial query tile: per-thread stores of the valid rows (a box would spill into the
      // next sequence's rows)
      __nv_bfloat16* dst = a.out + static_cast<long long>(s.q0 + (row_valid ? row_j : 0)) * a.out_stride +
                           (2 * h + row_g) * kHeadDim;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(tmem + kTwOCol + lane_base + c * 32, ov);
        tc_wait_ld();
        if (row_valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack_bf16x2(ov[i] * inv, ov[i + 1] * inv);
            w.y = pack_bf16x2(ov[i + 2] * inv, ov[i + 3] * inv);
            w.z = pack_bf16x2(ov[i + 4] * inv, ov[i + 5] * inv);
            w.w = pack_bf16x2(ov[i + 6] * inv, ov[i + 7] * inv);
            reinterpret_cast<uint4*>(dst + c * 32 + i)[0] = w;
          }
        }
      }
    }
  }

  // ------------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    // a role gave up: let the copies and MMAs already in flight finish (bounded) before TMEM and shared memory go away
    if (tid == kTwMmaWarp * 32) {
      umma_commit(&bars[TwSmem::kFinal]);
      mbar_wait_bounded(&bars[TwSmem::kFinal], 0, 200000000ull);
    }
    if (tid == 0) {                                           // the P.V issuer
      umma_commit(&bars[TwSmem::kFinalPv]);
      mbar_wait_bounded(&bars[TwSmem::kFinalPv], 0, 200000000ull);
    }
    if (tid == kTwProducerWarp * 32) {
      mbar_wait_bounded(&bars[TwSmem::kQFull], 0, 200000000ull);
      for (int is_v = 0; is_v < 2; ++is_v) {
        const int n = is_v ? *issued_v : *issued_k;
        for (int st = 0; st < 2; ++st) {
          const int last = (n - 1 - st) >= 0 ? ((n - 1 - st) & ~1) + st : -1;   // last tile issued into slot st
          if (last >= 0)
            mbar_wait_bounded(&bars[(is_v ? TwSmem::kVFull : TwSmem::kKFull) + st], (last >> 1) & 1, 200000000ull);
        }
      }
    }
  }
  __syncthreads();
  tc_fence_after();
  if (warp == kTwMmaWarp) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTwTmemCols));
  }
}

// ---------------------------------------------------------------- host side
// 3-D map over rows of `heads` x 128 bf16 (heads 256 bytes apart, rows row_bytes apart); box = 64 dims x 1 head x
// box_rows rows, 128-byte swizzle, zero fill past the last row.
bool make_rows_map(CUtensorMap* m, const void* base, long long rows, int heads, long long row_bytes, int box_rows) {
  const EncodeTiled enc = tensor_map_encoder();
  if (!enc || rows <= 0 || rows > (1ll << 31) - 1) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(heads),
                              static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadBytes), static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[3] = {64u, 1u, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// The warp-specialised kernel when the call fits it: row counts known, strides in whole 16-byte units, a positive
// softmax scale, and, with a prefix, page sizes whose boxes tile a 64-key tile (8, 16, 32 or a multiple of 64 tokens). Otherwise *launched stays
// false and the caller runs prefill_kernel.
cudaError_t launch_prefill_tma(const PrefillArgs& a, cudaStream_t stream, bool* launched) {
  *launched = false;
  if (a.q_rows <= 0 || a.kv_rows <= 0 || (a.q_stride * 2) % 16 || (a.kv_stride * 2) % 16 || !(a.scale_log2 > 0.f))
    return cudaSuccess;
  PfTmaParams p;
  memset(&p, 0, sizeof(p));
  p.a = a;
  if ((a.out_stride * 2) % 16 || !make_rows_map(&p.to, a.out, a.q_rows, kQHeads, a.out_stride * 2, 64) ||
      !make_rows_map(&p.tq, a.q, a.q_rows, kQHeads, a.q_stride * 2, 64) ||
      !make_rows_map(&p.tk, a.k, a.kv_rows, kKvHeads, a.kv_stride * 2, 64) ||
      !make_rows_map(&p.tv, a.v, a.kv_rows, kKvHeads, a.kv_stride * 2, 64))
    return cudaSuccess;
  // pool maps: needed to read a prefix (else the call does not fit this kernel) and used for the page writes
  const int ps = a.page_size;
  const bool box_ok = ps > 0 && (ps % 64 == 0 || ps == 8 || ps == 16 || ps == 32);
  p.box_rows = box_ok ? (ps >= 64 ? 64 : ps) : 64;
  p.pool_maps = 0;
  if ((a.prefix_lens != nullptr || a.write_kv) && box_ok) {
    const long long rows = static_cast<long long>(a.num_pages) * ps;
    p.pool_maps = make_rows_map(&p.tkp, a.k_pool, rows, kKvHeads, kRowBytes, p.box_rows) &&
                  make_rows_map(&p.tvp, a.v_pool, rows, kKvHeads, kRowBytes, p.box_rows);
  }
  if (a.prefix_lens != nullptr && !p.pool_maps) return cudaSuccess;
  static bool configured[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    e = cudaFuncSetAttribute(prefill_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TwSmem::kAlloc);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int qtiles = a.max_seqlen_q > 0 ? (a.max_seqlen_q + 63) / 64 : 1;
  prefill_tma_kernel<<<dim3(a.num_seqs, kKvHeads, qtiles), kTwThreads, TwSmem::kAlloc, stream>>>(p);
  *launched = true;
  return cudaGetLastError();
}

}  // namespace q3
