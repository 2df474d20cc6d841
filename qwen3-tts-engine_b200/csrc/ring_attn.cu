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
// One CTA per (stream, head): ring and chunk rows staged in shared memory (16-byte loads), scores and softmax in fp32.
#include "q3_common.cuh"
#include "q3_kernels.h"

#include <cuda_fp16.h>

namespace q3 {

constexpr int kRingThreads = 128;

__device__ __forceinline__ float round_fp16(float x) { return __half2float(__float2half_rn(x)); }

template <int HD>
__global__ void __launch_bounds__(kRingThreads) ring_attn_kernel(const RingArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int b = blockIdx.x, hh = blockIdx.y, tid = threadIdx.x;
  const int n = a.n, RING = a.ring, NK = RING + n;
  constexpr int CH = HD / 8;                                 // 16-byte chunks per row
  __half* sK = reinterpret_cast<__half*>(smem);              // [RING + n][HD]: ring rows, then the chunk's rows
  __half* sV = sK + static_cast<size_t>(NK) * HD;
  __half* sQ = sV + static_cast<size_t>(NK) * HD;            // [n][HD]
  float* sS = reinterpret_cast<float*>(sQ + n * HD);         // [n][RING + n] scores, then P
  float* sR = sS + n * NK;                                   // [kRingThreads][2] partial P.V sums of the ring keys

  const long long row = a.ring_rows[b];
  const long long pos = a.pos[b];
  const __half* kr = a.k_ring + row * a.ring_stream_stride + hh * HD;
  const __half* vr = a.v_ring + row * a.ring_stream_stride + hh * HD;
  // every row is staged with asynchronous 16-byte copies, all in flight together
  for (int i = tid; i < RING * CH; i += kRingThreads) {
    const int j = i / CH, c = i - j * CH;
    cp_async16(sK + j * HD + c * 8, kr + j * a.ring_slot_stride + c * 8);
    cp_async16(sV + j * HD + c * 8, vr + j * a.ring_slot_stride + c * 8);
  }
  for (int i = tid; i < n * CH; i += kRingThreads) {
    const int f = i / CH, c = i - f * CH;
    const long long off = b * a.qkv_batch_stride + f * a.qkv_frame_stride + hh * HD + c * 8;
    cp_async16(sK + (RING + f) * HD + c * 8, a.k_new + off);
    cp_async16(sV + (RING + f) * HD + c * 8, a.v_new + off);
    cp_async16(sQ + f * HD + c * 8, a.q + off);
  }
  cp_async_wait_all();
  __syncthreads();

  // ---- scores: fp16-rounded dot products, scaled and masked in fp32. Slot j holds frame qj = (pos-1) - d with
  //      d = ((pos-1) - j) mod RING; "qj >= 0 and qj >= pos + i - PAST" is "d <= min(pos-1, PAST-1-i)".
  const long long pm1 = pos - 1;
  const int pm1_mod = static_cast<int>(((pm1 % RING) + RING) % RING);
  const int d_cap = pm1 < 0 ? -1 : static_cast<int>(pm1 < 0x7fffffff ? pm1 : 0x7fffffff);
  for (int p = tid; p < n * NK; p += kRingThreads) {
    const int i = p / NK, j = p - i * NK;
    bool ok;
    if (j < RING) {
      int d = pm1_mod - j;
      if (d < 0) d += RING;
      ok = d <= d_cap && d <= a.past - 1 - i;
    } else {
      ok = (j - RING) <= i;
    }
    float s = -INFINITY;
    if (ok) {
      // lanes score consecutive keys whose rows sit a multiple of 32 banks apart: each starts at word j, so the 32
      // lanes of a warp read 32 distinct banks
      const __half2* qh = reinterpret_cast<const __half2*>(sQ + i * HD);
      const __half2* kh = reinterpret_cast<const __half2*>(sK + j * HD);
      float acc = 0.f;
#pragma unroll 8
      for (int e = 0; e < HD / 2; ++e) {
        const int w = (e + j) & (HD / 2 - 1);
        const float2 q2 = __half22float2(qh[w]), k2 = __half22float2(kh[w]);
        acc = fmaf(q2.x, k2.x, acc);
        acc = fmaf(q2.y, k2.y, acc);
      }
      s = round_fp16(acc) * a.scale;
    }
    sS[i * NK + j] = s;
  }
  __syncthreads();

  // ---- softmax per query row (one warp per row), P rounded to fp16
  const int warp = tid >> 5, lane = tid & 31;
  for (int i = warp; i < n; i += kRingThreads / 32) {
    float* srow = sS + i * NK;
    float m = -INFINITY;
    for (int j = lane; j < NK; j += 32) m = fmaxf(m, srow[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
    for (int j = lane; j < NK; j += 32) {
      const float e = srow[j] == -INFINITY ? 0.f : expf(srow[j] - m);
      srow[j] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.f / sum;                             // the query always sees itself: sum > 0
    for (int j = lane; j < NK; j += 32) srow[j] = round_fp16(srow[j] * inv);
  }
  __syncthreads();

  // ---- o = fp16(fp16(P_ring V_ring) + fp16(P_new V_new)), two dims per task; when the chunk has fewer tasks than
  //      threads, the ring keys are split into G groups whose partial sums are added in group order
  const int tasks = n * (HD / 2);
  const int G = tasks >= kRingThreads ? 1 : kRingThreads / tasks;
  for (int p = tid; p < tasks * G; p += kRingThreads) {
    const int g = p / tasks, t = p - g * tasks;
    const int i = t / (HD / 2), d2 = t - i * (HD / 2);
    const float* prow = sS + i * NK;
    float r0 = 0.f, r1 = 0.f;
    const int j0 = g * RING / G, j1 = (g + 1) * RING / G;
    for (int j = j0; j < j1; ++j) {
      const float pj = prow[j];
      if (pj == 0.f) continue;                               // masked slot: never read its (possibly stale) V
      const float2 v = __half22float2(reinterpret_cast<const __half2*>(sV + j * HD)[d2]);
      r0 = fmaf(pj, v.x, r0);
      r1 = fmaf(pj, v.y, r1);
    }
    if (G > 1) {
      sR[2 * p] = r0;
      sR[2 * p + 1] = r1;
    } else {
      float n0 = 0.f, n1 = 0.f;
      for (int j = RING; j < NK; ++j) {
        const float pj = prow[j];
        const float2 v = __half22float2(reinterpret_cast<const __half2*>(sV + j * HD)[d2]);
        n0 = fmaf(pj, v.x, n0);
        n1 = fmaf(pj, v.y, n1);
      }
      const __half2 o = __floats2half2_rn(round_fp16(r0) + round_fp16(n0), round_fp16(r1) + round_fp16(n1));
      reinterpret_cast<__half2*>(a.out + b * a.out_batch_stride + i * a.out_frame_stride + hh * HD)[d2] = o;
    }
  }
  if (G > 1) {                                               // uniform across the CTA
    __syncthreads();
    for (int t = tid; t < tasks; t += kRingThreads) {
      const int i = t / (HD / 2), d2 = t - i * (HD / 2);
      const float* prow = sS + i * NK;
      float r0 = 0.f, r1 = 0.f, n0 = 0.f, n1 = 0.f;
      for (int g = 0; g < G; ++g) {
        r0 += sR[2 * (g * tasks + t)];
        r1 += sR[2 * (g * tasks + t) + 1];
      }
      for (int j = RING; j < NK; ++j) {
        const float pj = prow[j];
        const float2 v = __half22float2(reinterpret_cast<const __half2*>(sV + j * HD)[d2]);
        n0 = fmaf(pj, v.x, n0);
        n1 = fmaf(pj, v.y, n1);
      }
      const __half2 o = __floats2half2_rn(round_fp16(r0) + round_fp16(n0), round_fp16(r1) + round_fp16(n1));
      reinterpret_cast<__half2*>(a.out + b * a.out_batch_stride + i * a.out_frame_stride + hh * HD)[d2] = o;
    }
  }

  // ---- the chunk's columns into the ring (slots of frames outside every window of this launch; read above)
  if (a.write_new) {
    __half* kw = a.k_ring + row * a.ring_stream_stride + hh * HD;
    __half* vw = a.v_ring + row * a.ring_stream_stride + hh * HD;
    for (int i = tid; i < n * CH; i += kRingThreads) {
      const int f = i / CH, c = i - f * CH;
      const long long slot = (pos + f) % RING;
      reinterpret_cast<uint4*>(kw + slot * a.ring_slot_stride)[c] = reinterpret_cast<const uint4*>(sK + (RING + f) * HD)[c];
      reinterpret_cast<uint4*>(vw + slot * a.ring_slot_stride)[c] = reinterpret_cast<const uint4*>(sV + (RING + f) * HD)[c];
    }
  }
}

size_t ring_smem_bytes(int ring, int hd, int n) {
  return (2ull * (ring + n) + n) * hd * sizeof(__half) + static_cast<size_t>(n) * (ring + n) * sizeof(float) +
         2ull * kRingThreads * sizeof(float);
}

cudaError_t launch_ring_attn(const RingArgs& a, cudaStream_t stream) {
  // the shared-memory limit is raised once per device, for the largest ring supported (kRingMaxSlots), so a call
  // made during stream capture sets no attribute
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(ring_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(ring_smem_bytes(kRingMaxSlots, 64, kRingMaxChunk)));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(ring_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(ring_smem_bytes(kRingMaxSlots, 128, kRingMaxChunk)));
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  if (a.B == 0 || a.n == 0) return cudaSuccess;
  const size_t bytes = ring_smem_bytes(a.ring, a.hd, a.n);
  dim3 grid(a.B, a.H);
  if (a.hd == 64)
    ring_attn_kernel<64><<<grid, kRingThreads, bytes, stream>>>(a);
  else
    ring_attn_kernel<128><<<grid, kRingThreads, bytes, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace q3
