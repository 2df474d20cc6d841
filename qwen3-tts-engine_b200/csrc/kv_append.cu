// K/V row append into a paged pool, bit-exact placement, sm_100a.
//
// Replaces the appends of the engine:
//   kc[l].view(-1, nkv, hd).index_copy_(0, slot, k)   engine/talker.py:72-73 (decode), 161-162 (packed prefill),
//                                                     engine/arrivals.py:144-145 (prefix + new rows)
// Two addressing modes: a flat destination row per input row (exactly index_copy_'s slot), or (seat, position)
// resolved through the block table: row = block_table[seat, pos / page] * page + pos % page.
// Each thread moves 16 bytes; consecutive threads cover consecutive bytes of a row, so loads and stores are coalesced.
#include "q3_common.cuh"
#include "q3_kernels.h"

namespace q3 {

__global__ void __launch_bounds__(256) kv_append_kernel(const AppendArgs a) {
  const int vec_per_row = a.row_elems / 8;                 // 16-byte vectors per row
  const long long total = 2ll * a.n_rows * vec_per_row;    // K and V
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long rv = idx / vec_per_row;
    const int vec = static_cast<int>(idx - rv * vec_per_row);
    const int which = static_cast<int>(rv & 1);            // 0: K, 1: V (interleaved so a warp's 512 B stay in one row)
    const int row = static_cast<int>(rv >> 1);
    long long dst;
    if (a.slots != nullptr) {
      dst = a.slots[row];
    } else {
      const int seat = a.seat_of_row != nullptr ? a.seat_of_row[row] : row;
      const int pos = a.positions[row];
      const int pidx = pos / a.page_size;
      if (pos < 0 || pidx >= a.max_pages) {
        if (vec == 0) atomicOr(a.status, kStatusBadLength);
        continue;
      }
      const int pg = a.block_table[static_cast<long long>(seat) * a.bt_stride + pidx];
      dst = static_cast<long long>(pg) * a.page_size + (pos - pidx * a.page_size);
    }
    if (dst < 0 || dst >= a.pool_rows) {
      if (vec == 0) atomicOr(a.status, kStatusBadPage);
      continue;
    }
    const __nv_bfloat16* src = (which ? a.v_rows : a.k_rows) + static_cast<long long>(row) * a.rows_stride;
    __nv_bfloat16* pool = which ? a.v_pool : a.k_pool;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + vec);
    reinterpret_cast<uint4*>(pool + dst * a.row_elems)[vec] = v;
  }
}

// Shared-prefix copy at admission. engine/arrivals.py:67-96 computes, once per (voice, language), the K/V of the k
// prompt positions every request of that voice shares (pK/pV [layers, slots, k, 8, 128]); arrivals.py:139-145 writes
// them into each admitted seat (positions 0..k-1) together with the new rows. Here all layers, seats and prefix rows go
// in one launch: vector `idx` -> (layer, batch row, prefix row, K or V, 16-byte vector), destination through the block
// table of the seat, pool of the layer read from a device array of per-layer pool addresses.
__global__ void __launch_bounds__(256) kv_copy_prefix_kernel(const PrefixCopyArgs a) {
  const int vec_per_row = a.row_elems / 8;
  const long long per_b = 2ll * a.prefix_len * vec_per_row;
  const long long total = static_cast<long long>(a.L) * a.B * per_b;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long lb = idx / per_b;
    long long rem = idx - lb * per_b;
    const int l = static_cast<int>(lb / a.B), b = static_cast<int>(lb - static_cast<long long>(l) * a.B);
    const long long rv = rem / vec_per_row;
    const int vec = static_cast<int>(rem - rv * vec_per_row);
    const int which = static_cast<int>(rv & 1);
    const int r = static_cast<int>(rv >> 1);
    const int pidx = r / a.page_size;
    if (pidx >= a.max_pages) {
      if (vec == 0) atomicOr(a.status, kStatusBadLength);
      continue;
    }
    const long long seat = a.seat[b];
    const int pg = a.block_table[seat * a.bt_stride + pidx];
    const long long dst = static_cast<long long>(pg) * a.page_size + (r - pidx * a.page_size);
    if (pg < 0 || dst >= a.pool_rows) {
      if (vec == 0) atomicOr(a.status, kStatusBadPage);
      continue;
    }
    const __nv_bfloat16* src = (which ? a.v_src : a.k_src) + l * a.src_layer_stride + a.slot[b] * a.src_slot_stride +
                               static_cast<long long>(r) * a.row_elems;
    __nv_bfloat16* pool = reinterpret_cast<__nv_bfloat16*>(which ? a.v_pools[l] : a.k_pools[l]);
    reinterpret_cast<uint4*>(pool + dst * a.row_elems)[vec] = __ldg(reinterpret_cast<const uint4*>(src) + vec);
  }
}

cudaError_t launch_kv_copy_prefix(const PrefixCopyArgs& a, int num_sms, cudaStream_t stream) {
  const long long total = 2ll * a.L * a.B * a.prefix_len * (a.row_elems / 8);
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  const long long cap = static_cast<long long>(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  kv_copy_prefix_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_kv_append(const AppendArgs& a, int num_sms, cudaStream_t stream) {
  const long long total = 2ll * a.n_rows * (a.row_elems / 8);
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  const long long cap = static_cast<long long>(num_sms) * 8;
  if (blocks > cap) blocks = cap;
  kv_append_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace q3
