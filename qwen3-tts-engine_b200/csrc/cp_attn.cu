// Code-predictor attention step, sm_100a: one query token over a per-seat 16-slot K/V cache, GQA 16/8, head_dim 128.
//
// Replaces, per (step, layer) of CodePredictor._s (engine/code_predictor.py:52-60):
//   K.index_copy_(2, [p], k); V.index_copy_(2, [p], v)                  engine/code_predictor.py:58
//   att = q.view(B,8,2,128) @ K^T * scale + mask[p]; softmax; @ V       engine/code_predictor.py:46-47
// with fp32 scores and softmax as in the reference's intended kernel cp_attn (engine/cp_attn.py:14-30), but fp32
// probabilities into P.V (cp_attn.py rounds them to bf16), fp32 accumulation, bf16 output. Slots >= n_live are not read.
//
// Two CTAs per seat (KV heads 0-3 and 4-7), one warp per KV head; lane l owns dims 4l..4l+3 of both q heads of the
// group. The live K and V rows are staged in shared memory by copies issued up front (one round of memory latency, no
// registers held), sized by n_live, so the grid of 2 x batch small CTAs runs in about one wave: one TMA bulk copy per
// (head, K/V) when the slot rows of a head are one contiguous, 16-byte aligned range (the engine's [B, 8, 16, 128]
// caches), else 8-byte asynchronous copies per lane. With k_new
// given, the new row is stored to slot n_live-1 and used from registers. With the norm weights given (q3_cp_step_qkv,
// the kernel instantiated with FUSE), q and k_new are raw projections: both q heads and the new k row get RMSNorm +
// RoPE here (code_predictor.py:40-41).
#include "q3_common.cuh"
#include "q3_kernels.h"

namespace q3 {

constexpr int kCpWarps = 4;   // KV heads per CTA: a seat takes two CTAs

// Shared memory of one CTA for n live slots: per warp K and V pieces [n][32 lanes] of 8 bytes (row-major [n][128]
// bf16), then P [32] floats per warp, then one mbarrier per warp.
__host__ __device__ constexpr size_t cp_smem_bytes(int n) {
  return static_cast<size_t>(kCpWarps) * (2 * n * 256 + 32 * sizeof(float) + sizeof(uint64_t));
}

__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(smem_dst)), "l"(gsrc) : "memory");
}

template <bool FUSE>
__global__ void __launch_bounds__(kCpWarps * 32) cp_attn_kernel(const CpArgs a) {
  extern __shared__ __align__(16) uint8_t cp_smem[];
  const int b = blockIdx.x, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y * kCpWarps + w;
  const int n = a.n_live, pnew = n - 1;
  const bool append = a.k_new != nullptr;
  uint2* sK = reinterpret_cast<uint2*>(cp_smem) + w * (2 * n * 32);   // [slot][lane]: dims 4l..4l+3 of head h
  uint2* sV = sK + n * 32;
  float* pbuf = reinterpret_cast<float*>(cp_smem + static_cast<size_t>(kCpWarps) * 2 * n * 256) + w * 32;
  uint64_t* bar = reinterpret_cast<uint64_t*>(cp_smem + static_cast<size_t>(kCpWarps) * (2 * n * 256 + 128)) + w;

  // ---- the live K/V slots of head h (all but the appended one), in flight while q / k_new load and the fused norm +
  //      RoPE run: one bulk copy each for K and V, or asynchronous 8-byte copies (one 256-byte row per warp
  //      instruction)
  const __nv_bfloat16* kb = a.K + static_cast<long long>(b) * a.sk_b + h * a.sk_h + 4 * lane;
  const __nv_bfloat16* vb = a.V + static_cast<long long>(b) * a.sv_b + h * a.sv_h + 4 * lane;
  const int n_copy = append ? n - 1 : n;
  if (a.bulk) {
    if (lane == 0 && n_copy > 0) {
      mbar_init(bar, 1);
      fence_mbar_init();
      mbar_arrive_expect_tx(bar, static_cast<uint32_t>(2 * n_copy * kHeadBytes));
      bulk_g2s(sK, kb, n_copy * kHeadBytes, bar);
      bulk_g2s(sV, vb, n_copy * kHeadBytes, bar);
    }
  } else {
    for (int s = 0; s < n_copy; ++s) {
      cp_async8(sK + s * 32 + lane, kb + s * a.sk_s);
      cp_async8(sV + s * 32 + lane, vb + s * a.sv_s);
    }
  }
  const __nv_bfloat16* qp = a.q + static_cast<long long>(b) * a.q_stride + (2 * h) * kHeadDim + 4 * lane;
  float4 q0 = bf16x4_to_float4(*reinterpret_cast<const uint2*>(qp));
  float4 q1 = bf16x4_to_float4(*reinterpret_cast<const uint2*>(qp + kHeadDim));
  uint2 kn = make_uint2(0, 0), vn = make_uint2(0, 0);
  if (append) {
    const long long off = static_cast<long long>(b) * a.kv_new_stride + h * kHeadDim + 4 * lane;
    kn = *reinterpret_cast<const uint2*>(a.k_new + off);
    vn = *reinterpret_cast<const uint2*>(a.v_new + off);
  }
  if constexpr (FUSE) {   // fused q/k RMSNorm + RoPE
    const long long ro = static_cast<long long>(b) * a.rope_stride;
    const __nv_bfloat16* cs = a.rope_cos + ro;
    const __nv_bfloat16* sn = a.rope_sin + ro;
    q0 = rms_rope_head(q0, a.qn_w, cs, sn, a.eps, lane);
    q1 = rms_rope_head(q1, a.qn_w, cs, sn, a.eps, lane);
    kn = float4_to_bf16x4(rms_rope_head(bf16x4_to_float4(kn), a.kn_w, cs, sn, a.eps, lane));
  }
  if (append) {
    sK[pnew * 32 + lane] = kn;
    sV[pnew * 32 + lane] = vn;
    *reinterpret_cast<uint2*>(const_cast<__nv_bfloat16*>(kb) + pnew * a.sk_s) = kn;
    *reinterpret_cast<uint2*>(const_cast<__nv_bfloat16*>(vb) + pnew * a.sv_s) = vn;
  }
  if (a.bulk) {
    __syncwarp();   // the barrier's initialisation (lane 0) before any lane waits on it
    if (n_copy > 0 && !mbar_wait_bounded(bar, 0)) {
      // the copies did not land within the limit: flag it, leave the outputs untouched, and keep the shared memory
      // alive (bounded) until the copies in flight are done
      if (lane == 0) {
        atomicOr(a.status, kStatusWaitTimeout);
        mbar_wait_bounded(bar, 0, 100000000ull);
      }
      return;
    }
  } else {
    cp_async_wait_all();
  }
  __syncwarp();

  const float sl = a.scale_log2;
  q0.x *= sl; q0.y *= sl; q0.z *= sl; q0.w *= sl;
  q1.x *= sl; q1.y *= sl; q1.z *= sl; q1.w *= sl;
  float sc[32];
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    if (s < n) {
      const float4 k = bf16x4_to_float4(sK[s * 32 + lane]);
      sc[s] = q0.x * k.x + q0.y * k.y + q0.z * k.z + q0.w * k.w;
      sc[16 + s] = q1.x * k.x + q1.y * k.y + q1.z * k.z + q1.w * k.w;
    } else {
      sc[s] = 0.f;
      sc[16 + s] = 0.f;
    }
  }
  const float x0 = transpose_reduce<32>(sc, lane);   // lane l: q head (l >> 4) of the group, slot (l & 15)
  const bool valid = (lane & 15) < n;
  const float x = valid ? x0 : -INFINITY;
  float m = x;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float p = valid ? exp2f(x - m) : 0.f;
  float sum = p;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  // P stays fp32 for P.V. engine/cp_attn.py:26-27 (and the bf16 matmul of code_predictor.py:47) round it to the model
  // dtype first; keeping it costs nothing here (it lives in registers / shared memory either way) and removes that
  // rounding from the error against the reference's fp32 result (the scores are fp32 dot products for the same reason).
  p = p / sum;
  pbuf[lane] = p;
  __syncwarp();

  float4 o0 = make_float4(0, 0, 0, 0), o1 = o0;
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    if (s < n) {
      const float p0 = pbuf[s], p1 = pbuf[16 + s];
      const float4 v = bf16x4_to_float4(sV[s * 32 + lane]);
      o0.x += p0 * v.x; o0.y += p0 * v.y; o0.z += p0 * v.z; o0.w += p0 * v.w;
      o1.x += p1 * v.x; o1.y += p1 * v.y; o1.z += p1 * v.z; o1.w += p1 * v.w;
    }
  }
  __nv_bfloat16* op = a.out + static_cast<long long>(b) * a.out_stride + (2 * h) * kHeadDim + 4 * lane;
  *reinterpret_cast<uint2*>(op) = float4_to_bf16x4(o0);
  *reinterpret_cast<uint2*>(op + kHeadDim) = float4_to_bf16x4(o1);
}

cudaError_t launch_cp_attn(const CpArgs& a, cudaStream_t stream) {
  if (a.B == 0) return cudaSuccess;
  const dim3 grid(a.B, kKvHeads / kCpWarps);
  const size_t bytes = cp_smem_bytes(a.n_live);
  if (a.qn_w != nullptr)
    cp_attn_kernel<true><<<grid, kCpWarps * 32, bytes, stream>>>(a);
  else
    cp_attn_kernel<false><<<grid, kCpWarps * 32, bytes, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace q3
