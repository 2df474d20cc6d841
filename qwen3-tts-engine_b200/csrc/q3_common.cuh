// Shared device helpers for the q3attn kernels (sm_100a only).
//
// Layout facts used everywhere (the engine's model family, engine/talker.py:26-31):
//   16 query heads, 8 KV heads (GQA group 2: q head h reads KV head h/2), head_dim 128, bf16 storage.
//   A KV pool is [num_pages, page_size, 8, 128] bf16: one token row holds all 8 KV heads = 2048 contiguous bytes, and
//   one KV head of a row is 256 contiguous bytes.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "q3attn kernels are written for sm_100a (B200) only"
#endif

namespace q3 {

constexpr int kHeadDim = 128;
constexpr int kKvHeads = 8;
constexpr int kGroup = 2;                       // q heads per KV head
constexpr int kQHeads = kKvHeads * kGroup;      // 16
constexpr int kRowBytes = kKvHeads * kHeadDim * 2;   // 2048: one token row, all KV heads
constexpr int kHeadBytes = kHeadDim * 2;             // 256: one KV head of one token row
constexpr float kLog2e = 1.4426950408889634f;

// Error bits a kernel may OR into its status word (read back by q3_read_status()).
enum : uint32_t {
  kStatusWaitTimeout = 1u << 0,   // an mbarrier wait gave up after its time limit
  kStatusBadPage = 1u << 1,       // a block-table entry outside [0, num_pages)
  kStatusBadLength = 1u << 2,     // a sequence length beyond the block table's capacity
};

// ---------------------------------------------------------------- bf16 <-> fp32
// Four bf16 packed in a uint2 -> four floats (a bf16 is the top half of an fp32).
__device__ __forceinline__ float4 bf16x4_to_float4(uint2 w) {
  float4 f;
  f.x = __uint_as_float(w.x << 16);
  f.y = __uint_as_float(w.x & 0xffff0000u);
  f.z = __uint_as_float(w.y << 16);
  f.w = __uint_as_float(w.y & 0xffff0000u);
  return f;
}

// Two bf16 packed in a uint32 (low half first) -> two floats.
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t x) {
  return make_float2(__uint_as_float(x << 16), __uint_as_float(x & 0xffff0000u));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint2 float4_to_bf16x4(float4 f) {
  return make_uint2(pack_bf16x2(f.x, f.y), pack_bf16x2(f.z, f.w));
}

__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// ---------------------------------------------------------------- q/k RMSNorm + rotate-half RoPE of one head
// One head of 128 dims held 4 dims per lane (lane l: dims 4l..4l+3), x = the raw head as floats (bf16 values).
// Arithmetic and rounding points of engine/ops.py:51-60 run in bf16:
//   xn  = bf16(x * rsqrt(mean(x^2) + eps))                      normalise in fp32, cast back     (ops.py:53-54)
//   y   = bf16(w * xn)                                                                          (ops.py:55)
//   out = bf16(bf16(y * cos) + bf16(rot(y) * sin)),  rot(y)[d] = -y[d + 64] (d < 64), y[d - 64]  (ops.py:58-60)
// Dims d and d + 64 live in lanes l and l + 16, so rot() is one shuffle. w, cs, sn point at [128] bf16 rows.
__device__ __forceinline__ float4 rms_rope_head(float4 x, const __nv_bfloat16* w, const __nv_bfloat16* cs,
                                               const __nv_bfloat16* sn, float eps, int lane) {
  float ss = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss * (1.f / kHeadDim) + eps);
  const float4 wv = bf16x4_to_float4(*reinterpret_cast<const uint2*>(w + 4 * lane));
  float4 y;
  y.x = round_bf16(wv.x * round_bf16(x.x * r));
  y.y = round_bf16(wv.y * round_bf16(x.y * r));
  y.z = round_bf16(wv.z * round_bf16(x.z * r));
  y.w = round_bf16(wv.w * round_bf16(x.w * r));
  const float sg = lane < 16 ? -1.f : 1.f;
  const float4 rt = make_float4(sg * __shfl_xor_sync(0xffffffffu, y.x, 16), sg * __shfl_xor_sync(0xffffffffu, y.y, 16),
                                sg * __shfl_xor_sync(0xffffffffu, y.z, 16), sg * __shfl_xor_sync(0xffffffffu, y.w, 16));
  const float4 c = bf16x4_to_float4(*reinterpret_cast<const uint2*>(cs + 4 * lane));
  const float4 s = bf16x4_to_float4(*reinterpret_cast<const uint2*>(sn + 4 * lane));
  return make_float4(round_bf16(round_bf16(y.x * c.x) + round_bf16(rt.x * s.x)),
                     round_bf16(round_bf16(y.y * c.y) + round_bf16(rt.y * s.y)),
                     round_bf16(round_bf16(y.z * c.z) + round_bf16(rt.z * s.z)),
                     round_bf16(round_bf16(y.w * c.w) + round_bf16(rt.w * s.w)));
}

// ---------------------------------------------------------------- shared-memory barriers and bulk copies
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before its later async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` of `bar` to complete, giving up after ~`limit_ns` (default 2 s). Returns false on timeout.
// No wait in these kernels is expected to take more than microseconds; the limit only turns a broken pipeline into an
// error status instead of a hung GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
#pragma unroll 1
  for (int i = 0; i < 4096; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
#pragma unroll 1
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

// 16-byte asynchronous copy global -> shared memory (no register staging; completion by cp_async_wait_all).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Close the group of this thread's asynchronous copies issued since the last commit.
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's committed copy groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// One-dimensional bulk copy global -> this CTA's shared memory, completion signalled on `bar` as transaction bytes.
// dst/src 16-byte aligned, bytes a multiple of 16 (the callers copy whole 2048-byte token rows).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ---------------------------------------------------------------- global loads
__device__ __forceinline__ uint2 ld_nc_u2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Reduce NV per-lane partial sums across the warp so that each lane ends with ONE complete sum.
// After the call v[0] of lane l holds the full sum of value index (l >> (5 - log2 NV)); e.g. NV = 32 -> index l,
// NV = 16 -> index l/2 (lane pairs hold the same total). Each halving step trades half the values with the partner lane.
template <int NV>
__device__ __forceinline__ float transpose_reduce(float (&v)[NV], int lane) {
  static_assert(NV >= 1 && NV <= 32 && (NV & (NV - 1)) == 0, "NV must be a power of two <= 32");
  int off = 16;
#pragma unroll
  for (int n = NV; n > 1; n >>= 1, off >>= 1) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = up ? v[i] : v[i + n / 2];
      const float keep = up ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
#pragma unroll
  for (; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
  return v[0];
}

}  // namespace q3
