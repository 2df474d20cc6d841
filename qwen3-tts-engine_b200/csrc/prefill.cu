// Prompt prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Replaces the prefill attention calls of the engine:
//   flash_attn_varlen_func(q, k, v, cu, cu, max, max, softmax_scale, causal=True)   engine/talker.py:169
//   flash_attn_func(q [S,R,16,128], K [S,k+R,8,128], V, softmax_scale, causal=True)  engine/arrivals.py:148
// and a chunked prefill whose cached prefix lives in the paged K/V pool, with the new rows written into the pages
// (the index_copy_ page writes of engine/talker.py:161-162 and engine/arrivals.py:144-145) by a second kernel of the
// same call (prefill_page_write_kernel).
//
// Sequence i has R_i query rows, N_i new key rows (N_i >= R_i) and P_i cached prefix keys in its pages; its L_i =
// P_i + N_i keys are indexed prefix first. Query j (0-based) sees keys 0 .. L_i - R_i + j (causal aligned to the bottom
// right, flash-attention's convention; with P = 0 and N = R it is the plain causal prefill).
//
// One CTA = (64-position query tile, KV head h, sequence). Its 128 accumulator rows are the 64 positions of q head 2h
// (rows 0-63) and of q head 2h+1 (rows 64-127): both heads share the K/V tiles. Per 64-key tile:
//   S[128 x 64]  = Q[128 x 128] K^T        8 x tcgen05.mma kind::f16 (M128 N64 K16), fp32 accumulator in TMEM
//   softmax                                 thread t owns TMEM lane t = accumulator row t (tcgen05.ld), no shuffles
//   O[128 x 128] += P[128 x 64] V[64 x 128]  4 x tcgen05.mma (M128 N128 K16), V as an MN-major operand, O in TMEM
// O is rescaled only when a row's running max grows by more than 2^8 (P then stays below 256, exact in fp32 sums and
// representable in bf16); the final division uses the same maxima, so the result is the exact softmax. Operands sit in
// shared memory in the canonical no-swizzle core-matrix layout (8 rows x 16 bytes per core matrix) described by the
// UMMA shared-memory descriptors below. A single thread issues the MMAs; tcgen05.commit arrives on an mbarrier that
// the other threads wait on (bounded waits).
#include "prefill_common.cuh"

namespace q3 {

constexpr int kPfThreads = 128;              // one warpgroup: thread t <-> TMEM lane t
constexpr int kPfQRows = 64;                 // query positions per tile (x 2 q heads = 128 MMA rows)
constexpr int kPfKeys = 64;                  // keys per tile
constexpr int kPfTmemCols = 256;             // S (64 columns) + O (128 columns), rounded to a power of two
constexpr uint32_t kPfSCol = 0, kPfOCol = 128;

struct PfSmem {
  static constexpr int kTile = kPfKeys * 256;                // one K (or V) tile: 64 keys x 128 dims, 16 KB
  static constexpr int kQ = 0;                               // 128 rows x 128 dims, K-major   32 KB
  static constexpr int kK = kQ + 128 * 256;                  // 2 x [64 keys x 128 dims], K-major (double buffer)
  static constexpr int kV = kK + 2 * kTile;                  // 2 x [128 dims x 64 keys], MN-major
  static constexpr int kP = kV + 2 * kTile;                  // 128 rows x 64 keys, K-major    16 KB
  static constexpr int kBar = kP + 128 * kPfKeys * 2;        // bar_s, bar_o
  static constexpr int kTmemSlot = kBar + 16;
  static constexpr int kBytes = kTmemSlot + 16;
};

// Shared-memory offsets of the canonical no-swizzle layouts (element = one bf16).
//   K-major [rows][128 or 64 k]: core matrix (8 rows x 8 k) = 128 contiguous bytes; k-chunks 128 B apart (LBO),
//   8-row groups `sbo` bytes apart (SBO).
__device__ __forceinline__ uint32_t kmajor_off(int row, int kchunk, int sbo) {
  return (row >> 3) * sbo + kchunk * 128 + (row & 7) * 16;
}
//   MN-major V [keys][128 dims] as the B operand (N = dims): core matrix (8 keys x 8 dims) = 128 bytes; key groups
//   128 B apart (LBO), 8-dim groups 1024 B apart (SBO).
__device__ __forceinline__ uint32_t v_off(int key, int dchunk) {
  return dchunk * 1024 + (key >> 3) * 128 + (key & 7) * 16;
}

__global__ void __launch_bounds__(kPfThreads, 1) prefill_kernel(const PrefillArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int h = blockIdx.y, seq = blockIdx.z;
  const PfSeq s = pf_seq(a, seq);
  const int ntq = s.R > 0 ? (s.R + kPfQRows - 1) / kPfQRows : 1;
  // the last query tiles see the most keys: they take the lowest block indices, so the heavy CTAs start first
  const int qt = ntq - 1 - static_cast<int>(blockIdx.x);
  if (qt < 0) return;                                        // uniform; nothing allocated yet

  if (s.R == 0) return;

  uint64_t* bar_s = reinterpret_cast<uint64_t*>(smem + PfSmem::kBar);
  uint64_t* bar_o = bar_s + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + PfSmem::kTmemSlot);
  const uint32_t sQ = smem_addr(smem + PfSmem::kQ), sK = smem_addr(smem + PfSmem::kK);
  const uint32_t sV = smem_addr(smem + PfSmem::kV), sP = smem_addr(smem + PfSmem::kP);

  if (warp == 0) {   // TMEM: 256 columns (at most two CTAs per SM fit by shared memory, so 512 columns suffice)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kPfTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    fence_mbar_init();
  }

  // ---- Q tile: thread t loads accumulator row t = (q head 2h + t/64, position 64*qt + t%64)
  const int row_g = tid >> 6, row_j = qt * kPfQRows + (tid & 63);
  const bool row_valid = row_j < s.R;
  {
    const uint4* src = reinterpret_cast<const uint4*>(a.q + static_cast<long long>(s.q0 + (row_valid ? row_j : 0)) * a.q_stride +
                                                      (2 * h + row_g) * kHeadDim);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint4 w = row_valid ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(smem + PfSmem::kQ + kmajor_off(tid, c, 2048)) = w;
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem + kPfSCol, t_o = tmem + kPfOCol;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;   // this warp's TMEM lanes

  const int L = s.P + s.Nn;
  const int shift = L - s.R;                                 // query j sees keys <= shift + j
  const int last_row = min(s.R - 1, qt * kPfQRows + kPfQRows - 1);
  const int key_end = a.causal ? min(L, shift + last_row + 1) : L;
  const int ntk = key_end > 0 ? (key_end + kPfKeys - 1) / kPfKeys : 0;
  const int my_limit = a.causal ? shift + row_j : L - 1;     // last visible key of this row

  constexpr uint32_t kIdescQK = umma_idesc_bf16(128, kPfKeys, 0, 0);
  constexpr uint32_t kIdescPV = umma_idesc_bf16(128, kHeadDim, 0, 1);
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;
  // K and V of a key tile: thread t holds half (t/64) of key kt*64 + t%64 in registers. The next tile's loads are
  // issued right after the current tile's Q K^T is issued, so they land while the tensor core and the softmax work.
  const int kk_local = tid & 63, half = tid >> 6;
  uint4 kreg[8], vreg[8];
  auto load_tile = [&](int kt) {
    const int kk = kt * kPfKeys + kk_local;
    const bool kv_ok = kt < ntk && kk < L;
    const uint4* ks = kv_ok ? reinterpret_cast<const uint4*>(pf_key_ptr(a, s, h, kk, 0)) + half * 8 : nullptr;
    const uint4* vs = kv_ok ? reinterpret_cast<const uint4*>(pf_key_ptr(a, s, h, kk, 1)) + half * 8 : nullptr;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      kreg[c] = kv_ok ? __ldg(ks + c) : make_uint4(0, 0, 0, 0);
      vreg[c] = kv_ok ? __ldg(vs + c) : make_uint4(0, 0, 0, 0);
    }
  };
  // Per key tile kt (K/V in buffer kt & 1): store the tile, one barrier, then a single thread issues O += P(kt-1) V(kt-1)
  // and S = Q K(kt)^T back to back under one commit. tcgen05.commit tracks every earlier MMA of the thread, so when
  // S(kt) is ready P(kt-1) V(kt-1) has finished too: P and O may then be rewritten, and the other K/V buffer (tile
  // kt-1) is free for tile kt+1. The last P V is issued after the loop.
  auto issue_pv = [&](int kt_pv) {
    const uint32_t vbuf = sV + (kt_pv & 1) * PfSmem::kTile;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
      umma_bf16(t_o, umma_smem_desc(sP + ks * 256, 128, 1024), umma_smem_desc(vbuf + ks * 256, 128, 1024), kIdescPV,
                (kt_pv > 0 || ks > 0) ? 1u : 0u);
  };
  load_tile(0);
  for (int kt = 0; kt < ntk && ok; ++kt) {
    const int buf = kt & 1;
    // ---- K and V tiles into buffer `buf` (its previous tile, kt-2, finished both MMAs)
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      *reinterpret_cast<uint4*>(smem + PfSmem::kK + buf * PfSmem::kTile + kmajor_off(kk_local, half * 8 + c, 2048)) =
          kreg[c];
      *reinterpret_cast<uint4*>(smem + PfSmem::kV + buf * PfSmem::kTile + v_off(kk_local, half * 8 + c)) = vreg[c];
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- O += P(kt-1) V(kt-1), then S = Q K(kt)^T
    if (tid == 0) {
      if (kt > 0) issue_pv(kt - 1);
      const uint32_t kbuf = sK + buf * PfSmem::kTile;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_bf16(t_s, umma_smem_desc(sQ + ks * 256, 128, 2048), umma_smem_desc(kbuf + ks * 256, 128, 2048), kIdescQK,
                  ks > 0 ? 1u : 0u);
      umma_commit(bar_s);
    }
    if (kt + 1 < ntk) load_tile(kt + 1);                     // in flight during this tile's MMAs and softmax
    if (!mbar_wait_bounded(bar_s, kt & 1)) {
      atomicOr(a.status, kStatusWaitTimeout);
      ok = false;
    }
    ok = __syncthreads_and(ok);                              // every thread leaves the loop together on a timeout
    if (!ok) break;
    tc_fence_after();
    // ---- softmax of this thread's row (exp2 domain, lazy max)
    float sv[2][32];
    tmem_ld32(t_s + lane_base, sv[0]);
    tmem_ld32(t_s + lane_base + 32, sv[1]);
    tc_wait_ld();
    // masking per element only on tiles that some row of the warp does not fully see (the causal diagonal, the last
    // keys); the maxima and sums run in 4 independent chains
    float cm4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    const int tile_last = kt * kPfKeys + kPfKeys - 1;
    if (__all_sync(0xffffffffu, row_valid && tile_last <= my_limit && tile_last < L)) {
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          sv[u][i] *= a.scale_log2;
          cm4[i & 3] = fmaxf(cm4[i & 3], sv[u][i]);
        }
    } else {
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int kk = kt * kPfKeys + u * 32 + i;
          const bool vis = row_valid ? (kk <= my_limit && kk < L) : (kk < L);
          sv[u][i] = vis ? sv[u][i] * a.scale_log2 : -INFINITY;
          cm4[i & 3] = fmaxf(cm4[i & 3], sv[u][i]);
        }
    }
    const float cmax = fmaxf(fmaxf(cm4[0], cm4[1]), fmaxf(cm4[2], cm4[3]));
    // the running max moves (and O is rescaled) only when it would grow by more than 8 (a factor 256 in P)
    const bool grow = cmax > m_run + 8.f || (m_run == -INFINITY && cmax > -INFINITY);
    const float m_new = grow ? cmax : m_run;
    const float alpha = grow ? exp2f(m_run - m_new) : 1.f;   // 0 on the first visible tile
    float ls4[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t pk[32];
    const float mm = m_new == -INFINITY ? 0.f : m_new;       // a row with nothing visible yet: every sv is -inf, p = 0
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float p0 = ex2_approx(sv[u][i] - mm);
        const float p1 = ex2_approx(sv[u][i + 1] - mm);
        ls4[(i >> 1) & 3] += p0 + p1;
        pk[u * 16 + i / 2] = pack_bf16x2(p0, p1);
      }
    const float lsum = (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
    l_run = l_run * alpha + lsum;
    m_run = m_new;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(smem + PfSmem::kP + kmajor_off(tid, c, 1024)) =
          make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    // ---- rescale O where a max moved (O holds tiles 0..kt-1, all finished; tile 0 starts O from zero instead)
    if (kt > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(t_o + lane_base + c * 32, ov);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] *= alpha;
        tmem_st32(t_o + lane_base + c * 32, ov);
      }
      tc_wait_st();
    }
  }
  // ---- the last O += P V
  if (ok && ntk > 0) {
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      issue_pv(ntk - 1);
      umma_commit(bar_o);
    }
    if (!mbar_wait_bounded(bar_o, 0)) {
      atomicOr(a.status, kStatusWaitTimeout);
      ok = false;
    }
    ok = __syncthreads_and(ok);
    tc_fence_after();
  }

  // ---- epilogue: O / l -> bf16 rows (a row that sees no key gets zeros, as flash-attention writes). The TMEM loads
  //      are warp-collective, so every thread takes part; only rows of the sequence store.
  if (ok) {
    __nv_bfloat16* dst = a.out + static_cast<long long>(s.q0 + (row_valid ? row_j : 0)) * a.out_stride +
                         (2 * h + row_g) * kHeadDim;
    const float inv = (ntk > 0 && l_run > 0.f) ? 1.f / l_run : 0.f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float ov[32];
      if (ntk > 0) {
        tmem_ld32(t_o + lane_base + c * 32, ov);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] = 0.f;
      }
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols));
  }
}

// The page writes of a chunked prefill (write_kv): new row r of sequence i goes to position P_i + r of its seat's pages,
// K and V, all 8 heads (2 KB per row each). A separate launch after the attention: the attention reads new keys from
// the input rows and only the prefix from the pages, so the order does not matter, and the writes then cost the
// attention CTAs nothing. CTA (x, i) walks sequence i's 16-byte vectors with a grid stride; loads are coalesced.
__global__ void __launch_bounds__(256) prefill_page_write_kernel(const PrefillArgs a) {
  const PfSeq s = pf_seq(a, blockIdx.y);
  constexpr int kVec = kKvHeads * kHeadDim / 8;              // 16-byte vectors per row and pool
  const long long total = 2ll * s.Nn * kVec;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(idx / (2 * kVec));
    const int rem = static_cast<int>(idx - static_cast<long long>(r) * 2 * kVec);
    const int which = rem / kVec, vec = rem - which * kVec;
    const long long prow = pf_pool_row(a, s.seat, s.P + r);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>((which ? a.v : a.k) + static_cast<long long>(s.k0 + r) * a.kv_stride) + vec);
    reinterpret_cast<uint4*>((which ? a.v_pool : a.k_pool) + prow * (kKvHeads * kHeadDim))[vec] = v;
  }
}

int g_prefill_kernel = 0;

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream) {
  if (a.num_seqs == 0) return cudaSuccess;
  bool launched = false;
  if (g_prefill_kernel == 0) {
    cudaError_t e = launch_prefill_tma(a, stream, &launched);
    if (e != cudaSuccess) return e;
  }
  if (launched) return cudaSuccess;                          // the TMA kernel does the page writes itself
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PfSmem::kBytes);
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  if (a.num_seqs == 0) return cudaSuccess;
  const int qtiles = a.max_seqlen_q > 0 ? (a.max_seqlen_q + kPfQRows - 1) / kPfQRows : 1;
  dim3 grid(qtiles, kKvHeads, a.num_seqs);
  prefill_kernel<<<grid, kPfThreads, PfSmem::kBytes, stream>>>(a);
  if (a.write_kv) prefill_page_write_kernel<<<dim3(16, a.num_seqs), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace q3
