// Paged decode attention with warp-level tensor-core MMAs for the per-chunk products, sm_100a.
//
// Same contract, work split and merge as paged_decode.cu (flat split-K over 8-token chunks, 8 warps = 8 KV heads per
// CTA, two CTAs per SM, TMA bulk copies refilled by the last warp to read a stage). What differs is how a warp turns
// a chunk into scores and outputs: 8 + 8 mma.sync.m16n8k16 (bf16 in, fp32 accumulate) and 16 ldmatrix instead of
// ~400 CUDA-core instructions per warp per chunk:
//   scores  S[g][t] = sum_d q[2h+g][d] K[t][d]     A = q (16 rows, rows 0-1 real), B = K^T via ldmatrix (t = n),
//                                                  8 k-steps of 16 dims; D rows 0-1 = the two q heads
//   output  O^T[d][g] += sum_t V[t][d] P[g][t]      A = V^T via ldmatrix.trans (16 dims x 8 tokens per tile),
//                                                  B = P straight from the score fragment (same lane layout),
//                                                  8 tiles of 16 dims
// The score fragment of lane l < 8 holds head l/4, tokens 2(l%4) and 2(l%4)+1 -- exactly the B-operand layout the
// output MMA wants for P, so probabilities never leave registers (rounded to bf16 for the MMA, as flash-attention
// does; the running sums stay fp32). Tensor-core throughput is irrelevant (the kernel is HBM-bound): the MMAs cut the
// instruction count per byte streamed.
//
// A stage is released as soon as its data is in registers -- K consumed by the score MMAs straight from shared memory,
// V moved into fragments -- before the softmax and the output MMAs, so the refill of the stage starts earlier and more
// chunks stay in flight per CTA. The q fragments are parked in the warp's shared relayout area between chunks so they
// occupy registers only during the score MMAs.
//
// ldmatrix reads 8 token rows at one column offset, so rows must not share a bank group: every token row is copied
// by its own 2 KB bulk copy into a stage row padded to 2064 bytes (row r starts on bank group r mod 8).
#include "decode_common.cuh"

namespace q3 {

constexpr int kPadRow = kRowBytes + 16;   // 2064: padded shared-memory token row

template <int NSTAGES>
struct MmaSmemLayout {
  static constexpr int kRows = 8;                                        // tokens per chunk
  static constexpr int kStageBytes = kRows * kPadRow;                    // K (or V) of one chunk
  static constexpr int kKOff = 0;
  static constexpr int kVOff = NSTAGES * kStageBytes;
  static constexpr int kOOff = ((2 * NSTAGES * kStageBytes + 15) / 16) * 16;   // per-warp [2][128] fp32 relayout
  static constexpr int kBarOff = kOOff + kDecodeWarps * 2 * kHeadDim * 4;       // full[NSTAGES]
  static constexpr int kDoneOff = kBarOff + NSTAGES * 8;                          // done[NSTAGES]
  static constexpr int kMiscOff = kDoneOff + ((NSTAGES * 4 + 15) / 16) * 16;
  static constexpr int kBytes = kMiscOff + 64;
};

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2_trans(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// D += A * B for one m16n8k16 tile.
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Copies of one chunk: lanes 0..7 copy K rows, lanes 8..15 the V rows, each 2 KB into its padded stage row. Called by
// a whole warp; lane 0 declares the transaction bytes first.
__device__ __forceinline__ void issue_chunk_rows(const DecodeArgs& a, const ChunkDesc& d, uint8_t* ks, uint8_t* vs,
                                                 uint64_t* bar, int lane) {
  if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(2 * d.rows * kRowBytes));
  __syncwarp();
  const int r = lane & 7;
  const bool is_v = (lane >> 3) & 1;
  if (lane < 16 && r < d.rows) {
    const __nv_bfloat16* src;
    if (r < d.pool_rows) {
      long long row;
      if (d.row0 >= 0) {
        row = d.row0 + r;
      } else {
        int room;
        row = pool_row_index(a, d.seat, d.tok0 + r, room);
      }
      src = (is_v ? a.v_pool : a.k_pool) + row * (kRowBytes / 2);
    } else {   // the appended token's row comes from k_new / v_new
      src = (is_v ? a.v_new : a.k_new) + static_cast<long long>(d.seat) * a.kv_new_stride;
    }
    fence_proxy_async_smem();
    bulk_g2s((is_v ? vs : ks) + r * kPadRow, src, kRowBytes, bar);
  }
}

template <int NSTAGES, int MIN_CTAS>
__global__ void __maxnreg__(decode_max_regs<MIN_CTAS>()) paged_decode_mma_kernel(const DecodeArgs a) {
  using SL = MmaSmemLayout<NSTAGES>;
  constexpr int ROWS = SL::kRows;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL::kBarOff);
  unsigned* done = reinterpret_cast<unsigned*>(smem + SL::kDoneOff);
  volatile int* abort_flag = reinterpret_cast<int*>(smem + SL::kMiscOff);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool append = a.k_new != nullptr;

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
  SeatCursor cur = plan.cur;

  // ---- prologue: warp 0 issues the first NSTAGES chunks; every warp keeps the descriptor of chunk i + NSTAGES
  SeatCursor look = cur;
  if (warp == 0) {
    for (int s = 0; s < NSTAGES && c0 + s < c1; ++s) {
      advance<ROWS>(a, look, c0 + s);
      issue_chunk_rows(a, make_desc<ROWS>(a, look, c0 + s), smem + SL::kKOff + s * SL::kStageBytes,
                       smem + SL::kVOff + s * SL::kStageBytes, &full[s], lane);
    }
  }
  look = cur;
  ChunkDesc nd{};
  if (c0 + NSTAGES < c1) {
    advance<ROWS>(a, look, c0 + NSTAGES);
    nd = make_desc<ROWS>(a, look, c0 + NSTAGES);
  }

  const int h = warp;
  const uint32_t ldsm_off = (lane & 7) * kPadRow + h * kHeadBytes + ((lane >> 3) & 1) * 16;   // this lane's row
  float* obuf = reinterpret_cast<float*>(smem + SL::kOOff) + warp * 2 * kHeadDim;
  const bool score_lane = lane < 8;               // lanes holding real scores: head lane/4, tokens 2(lane%4)+{0,1}
  const int t0 = 2 * (lane & 3);

  int it = 0;
  long long i = c0;
  bool aborted = false;
  while (i < c1 && !aborted) {
    advance<ROWS>(a, cur, i);
    // ---- q of this seat as A fragments: lane l < 8 holds row l/4 (q head 2h + l/4), dims 16ks + 2(l%4) (+8); parked
    //      in this warp's relayout area (unused until the seat ends) and re-read per chunk
    {
      // lanes >= 8 carry zero rows; their address is clamped onto heads 2h/2h+1 so no load leaves the q row
      const __nv_bfloat16* qrow =
          a.q + static_cast<long long>(cur.seat) * a.q_stride + (2 * h + ((lane >> 2) & 1)) * kHeadDim + t0;
      if (score_lane) {
        uint32_t w[16];
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          w[2 * ks] = __ldg(reinterpret_cast<const unsigned*>(qrow + 16 * ks));
          w[2 * ks + 1] = __ldg(reinterpret_cast<const unsigned*>(qrow + 16 * ks + 8));
        }
        uint4* dst = reinterpret_cast<uint4*>(obuf) + lane * 4;
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[e] = make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
      }
      __syncwarp();
    }
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;          // for head lane/4 (meaningful in lanes 0..7)
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
      const bool has_new = append && tok0 + rows == cur.len;
      uint8_t* kst = smem + SL::kKOff + stage * SL::kStageBytes;
      uint8_t* vst = smem + SL::kVOff + stage * SL::kStageBytes;
      const uint32_t kaddr = smem_addr(kst) + ldsm_off, vaddr = smem_addr(vst) + ldsm_off;

      // ---- scores straight from shared memory (two accumulation chains over the 8 k-steps)
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
      {
        uint32_t qa[16];
        const uint4* src = reinterpret_cast<const uint4*>(obuf) + (lane & 7) * 4;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint4 w = score_lane ? src[e] : make_uint4(0, 0, 0, 0);
          qa[4 * e] = w.x; qa[4 * e + 1] = w.y; qa[4 * e + 2] = w.z; qa[4 * e + 3] = w.w;
        }
#pragma unroll
        for (int ks = 0; ks < 8; ks += 2) {
          uint32_t b0, b1, c0r, c1r;
          ldsm_x2(kaddr + ks * 32, b0, b1);
          ldsm_x2(kaddr + (ks + 1) * 32, c0r, c1r);
          mma_bf16(sa, qa[2 * ks], 0u, qa[2 * ks + 1], 0u, b0, b1);
          mma_bf16(sb, qa[2 * ks + 2], 0u, qa[2 * ks + 3], 0u, c0r, c1r);
        }
      }
      // ---- V fragments (and the appended row) into registers, then release the stage
      uint32_t vf[8][2];
#pragma unroll
      for (int j = 0; j < 8; ++j) ldsm_x2_trans(vaddr + j * 32, vf[j][0], vf[j][1]);
      uint2 knew = make_uint2(0, 0), vnew = knew;
      if (has_new) {   // head h of the appended row, 4 dims per lane
        const int off = (h * kHeadDim + 4 * lane) * 2;
        knew = *reinterpret_cast<const uint2*>(kst + (rows - 1) * kPadRow + off);
        vnew = *reinterpret_cast<const uint2*>(vst + (rows - 1) * kPadRow + off);
      }
      __syncwarp();
      unsigned prev = 0;
      if (lane == 0) {
        __threadfence_block();   // this warp's shared-memory reads of the stage are done before the ticket
        prev = atomicAdd(&done[stage], 1u);
      }
      prev = __shfl_sync(0xffffffffu, prev, 0);
      if ((prev % kDecodeWarps) == kDecodeWarps - 1 && i + NSTAGES < c1) issue_chunk_rows(a, nd, kst, vst, &full[stage], lane);
      if (i + NSTAGES + 1 < c1) {   // descriptor (and block-table load) of the chunk this warp may issue next
        advance<ROWS>(a, look, i + NSTAGES + 1);
        nd = make_desc<ROWS>(a, look, i + NSTAGES + 1);
      }

      // ---- online softmax over the chunk's tokens
      const bool v0 = t0 < rows, v1 = t0 + 1 < rows;
      const float x0 = (score_lane && v0) ? (sa[0] + sb[0]) * a.scale_log2 : -INFINITY;
      const float x1 = (score_lane && v1) ? (sa[1] + sb[1]) * a.scale_log2 : -INFINITY;
      float cm = fmaxf(x0, x1);
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 1));
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 2));
      const float mn = score_lane ? fmaxf(m_run, cm) : 0.f;
      const float alpha = score_lane ? exp2f(m_run - mn) : 1.f;
      m_run = mn;
      const float p0 = (score_lane && v0) ? exp2f(x0 - mn) : 0.f;
      const float p1 = (score_lane && v1) ? exp2f(x1 - mn) : 0.f;
      l_run = l_run * alpha + p0 + p1;
      const uint32_t bp = score_lane ? pack_bf16x2(p0, p1) : 0u;

      // ---- rescale the outputs when a running max moved (lanes l%4 == 0 hold heads 0/1 in columns 0/1)
      const float al0 = __shfl_sync(0xffffffffu, alpha, 0), al1 = __shfl_sync(0xffffffffu, alpha, 4);
      if (__any_sync(0xffffffffu, (al0 != 1.f) || (al1 != 1.f))) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j][0] *= al0; o[j][1] *= al1; o[j][2] *= al0; o[j][3] *= al1;
        }
      }
      // ---- outputs: 8 tiles of 16 dims, A = V^T (tokens 0..7), B = P. In a partial chunk the rows past `rows` hold
      //      stale bytes; their halves of the V fragments are zeroed so no stale NaN/Inf pattern can reach the sums
      //      (lane l's fragments hold tokens 2(l%4) and 2(l%4)+1).
      const uint32_t vmask = (v0 ? 0x0000ffffu : 0u) | (v1 ? 0xffff0000u : 0u);
      const bool partial = rows < ROWS;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t a0 = vf[j][0], a1 = vf[j][1];
        if (partial) {
          a0 &= vmask;
          a1 &= vmask;
        }
        mma_bf16(o[j], a0, a1, 0u, 0u, bp, 0u);
      }

      // ---- fused append: this chunk holds the new token; write head h of its row into the pools
      if (has_new) {
        int room;
        const long long row = pool_row_index(a, cur.seat, cur.len - 1, room);
        const int off = h * kHeadDim + 4 * lane;
        *reinterpret_cast<uint2*>(a.k_pool + row * (kRowBytes / 2) + off) = knew;
        *reinterpret_cast<uint2*>(a.v_pool + row * (kRowBytes / 2) + off) = vnew;
      }
      if (*abort_flag) {
        aborted = true;
        break;
      }
    }   // chunks of this seat
    if (aborted) break;

    // ---- end of the seat's chunks in this CTA: sums and maxima of both heads, outputs relaid to 4 dims per lane
    float l = l_run;
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const float l0 = __shfl_sync(0xffffffffu, l, 0), l1 = __shfl_sync(0xffffffffu, l, 4);
    const float m0 = __shfl_sync(0xffffffffu, m_run, 0), m1 = __shfl_sync(0xffffffffu, m_run, 4);
    __syncwarp();   // every lane is done with the q fragments parked in obuf
    if ((lane & 3) == 0) {
      const int d = lane >> 2;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        obuf[j * 16 + d] = o[j][0];
        obuf[kHeadDim + j * 16 + d] = o[j][1];
        obuf[j * 16 + 8 + d] = o[j][2];
        obuf[kHeadDim + j * 16 + 8 + d] = o[j][3];
      }
    }
    __syncwarp();
    const float4 o0 = reinterpret_cast<const float4*>(obuf)[lane];
    const float4 o1 = reinterpret_cast<const float4*>(obuf + kHeadDim)[lane];
    __syncwarp();
    decode_finish_seat(a, plan, static_cast<int>(blockIdx.x), cur, h, lane, o0, o1, m0, m1, l0, l1);
  }

  // A warp that gave up may leave copies in flight into this CTA's shared memory: wait (bounded) for every issued
  // stage to land before the CTA exits.
  if (*abort_flag && lane == 0) {
    for (int j = 0; j < NSTAGES; ++j)
      mbar_wait_bounded(&full[(it + j) % NSTAGES], ((it + j) / NSTAGES) & 1, 100000000ull);
  }
}

template <int NSTAGES, int MIN_CTAS>
cudaError_t launch_decode_mma(const DecodeArgs& a, int grid, cudaStream_t stream) {
  using SL = MmaSmemLayout<NSTAGES>;
  auto kern = paged_decode_mma_kernel<NSTAGES, MIN_CTAS>;
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

template <int NSTAGES, int MIN_CTAS>
int occupancy_mma() {
  using SL = MmaSmemLayout<NSTAGES>;
  auto kern = paged_decode_mma_kernel<NSTAGES, MIN_CTAS>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SL::kBytes) != cudaSuccess) return -1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kDecodeThreads, SL::kBytes) != cudaSuccess) return -1;
  return n;
}

template cudaError_t launch_decode_mma<3, 2>(const DecodeArgs&, int, cudaStream_t);
template cudaError_t launch_decode_mma<2, 2>(const DecodeArgs&, int, cudaStream_t);
template int occupancy_mma<3, 2>();
template int occupancy_mma<2, 2>();

}  // namespace q3
