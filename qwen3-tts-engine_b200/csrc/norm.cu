// Row kernels around the attention layers, sm_100a: residual add + RMSNorm, SiLU-gated product, and the in-place q/k
// RMSNorm + RoPE of QKV projection rows. Each replaces a chain of small PyTorch ops (one launch each, ~8 for an
// RMSNorm, ~13 for a norm + RoPE) with one launch, keeping the reference's bf16 rounding points:
//   rms (engine/ops.py:51-55):      y = bf16(w * bf16(x * rsqrt(mean(x^2) + eps)))   (x = bf16(x + r) when r is given,
//                                   the residual add of talker.py:78-79 / code_predictor.py:48-50, written back to x)
//   mlp gate (engine/ops.py:63-65): y = bf16(bf16(silu(g)) * u)
//   q/k norm + RoPE (ops.py:51-60): rms_rope_head (q3_common.cuh), in place on the q and k heads of each row
// All three are memory-bound: one pass over the rows, 16-byte accesses, one warp per row (or head).
#include "q3_common.cuh"
#include "q3_kernels.h"

namespace q3 {

// One warp per row; lane l holds elements [l*8 + 256*j, +8) for j < H/256 (16-byte pieces, coalesced per j).
template <int H>
__global__ void __launch_bounds__(128) add_rms_norm_kernel(const RowNormArgs a) {
  constexpr int J = H / 256;
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  __nv_bfloat16* xr = a.x + row * a.x_stride;
  uint4 wv[J];   // the norm weight, loaded up front: its latency overlaps the row's loads and the reduction
#pragma unroll
  for (int j = 0; j < J; ++j) wv[j] = *reinterpret_cast<const uint4*>(a.w + 256 * j + 8 * lane);
  float v[J][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = 256 * j + 8 * lane;
    uint4 w = *reinterpret_cast<const uint4*>(xr + c);
    if (a.r != nullptr) {
      const uint4 rr = *reinterpret_cast<const uint4*>(a.r + row * a.r_stride + c);
      const uint32_t* xw = reinterpret_cast<const uint32_t*>(&w);
      const uint32_t* rw = reinterpret_cast<const uint32_t*>(&rr);
      uint4 s;
      uint32_t* sw = reinterpret_cast<uint32_t*>(&s);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 p = bf16x2_to_float2(xw[e]), q = bf16x2_to_float2(rw[e]);
        sw[e] = pack_bf16x2(p.x + q.x, p.y + q.y);      // the residual sum, rounded to bf16
      }
      w = s;
      *reinterpret_cast<uint4*>(xr + c) = s;
    }
    const uint32_t* ww = reinterpret_cast<const uint32_t*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 p = bf16x2_to_float2(ww[e]);
      v[j][2 * e] = p.x;
      v[j][2 * e + 1] = p.y;
      ss += p.x * p.x + p.y * p.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rs = rsqrtf(ss * (1.f / H) + a.eps);
  __nv_bfloat16* yr = a.y + row * a.y_stride;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = 256 * j + 8 * lane;
    const uint32_t* wwv = reinterpret_cast<const uint32_t*>(&wv[j]);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 g = bf16x2_to_float2(wwv[e]);
      ow[e] = pack_bf16x2(g.x * round_bf16(v[j][2 * e] * rs), g.y * round_bf16(v[j][2 * e + 1] * rs));
    }
    *reinterpret_cast<uint4*>(yr + c) = o;
  }
}

// y[row, c] = bf16(bf16(silu(g)) * u) with g = gu[row, c], u = gu[row, F + c]; 8 elements per thread.
__global__ void __launch_bounds__(256) silu_mul_kernel(const SiluMulArgs a) {
  const long long per_row = a.F / 8;
  const long long total = a.rows * per_row;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / per_row;
    const int c = static_cast<int>(i - row * per_row) * 8;
    const __nv_bfloat16* g = a.gu + row * a.gu_stride + c;
    const uint4 gv = *reinterpret_cast<const uint4*>(g);
    const uint4 uv = *reinterpret_cast<const uint4*>(g + a.F);
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
    const uint32_t* uw = reinterpret_cast<const uint32_t*>(&uv);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = bf16x2_to_float2(gw[e]), u = bf16x2_to_float2(uw[e]);
      const float s0 = round_bf16(x.x / (1.f + expf(-x.x))), s1 = round_bf16(x.y / (1.f + expf(-x.y)));
      ow[e] = pack_bf16x2(s0 * u.x, s1 * u.y);
    }
    *reinterpret_cast<uint4*>(a.y + row * a.y_stride + c) = o;
  }
}

// One warp per (row, head) of the 16 q + 8 k heads of a QKV row; norm + RoPE in place (v untouched).
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const QkNormRopeArgs a) {
  const int lane = threadIdx.x & 31;
  const long long wid = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  constexpr int kHeads = kQHeads + kKvHeads;
  if (wid >= a.rows * kHeads) return;
  const long long row = wid / kHeads;
  const int head = static_cast<int>(wid - row * kHeads);
  uint2* p = reinterpret_cast<uint2*>(a.qkv + row * a.qkv_stride + head * kHeadDim) + lane;
  const long long ro = row * a.rope_stride;
  const __nv_bfloat16* w = head < kQHeads ? a.qn_w : a.kn_w;
  *p = float4_to_bf16x4(rms_rope_head(bf16x4_to_float4(*p), w, a.rope_cos + ro, a.rope_sin + ro, a.eps, lane));
}

cudaError_t launch_add_rms_norm(const RowNormArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  const long long blocks = (a.rows + 3) / 4;
  switch (a.H) {
    case 1024: add_rms_norm_kernel<1024><<<static_cast<unsigned>(blocks), 128, 0, stream>>>(a); break;
    case 2048: add_rms_norm_kernel<2048><<<static_cast<unsigned>(blocks), 128, 0, stream>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const SiluMulArgs& a, int num_sms, cudaStream_t stream) {
  const long long total = a.rows * (a.F / 8);
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > static_cast<long long>(num_sms) * 16) blocks = static_cast<long long>(num_sms) * 16;
  silu_mul_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope(const QkNormRopeArgs& a, cudaStream_t stream) {
  const long long warps = a.rows * (kQHeads + kKvHeads);
  if (warps == 0) return cudaSuccess;
  qk_norm_rope_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace q3
