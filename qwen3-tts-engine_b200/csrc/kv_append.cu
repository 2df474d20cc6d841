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
