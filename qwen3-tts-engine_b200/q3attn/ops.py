"""PyTorch custom ops over the q3attn C ABI (torch.library.custom_op, opaque to torch.compile, graph-capturable).

Ops (namespace ``q3attn``):
  paged_decode(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, num_splits) -> out
  paged_decode_append(q, k, v, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, num_splits) -> out
      (mutates k_cache/v_cache: the new rows land at position cache_seqlens[b])
  kv_append_slots(k, v, k_cache, v_cache, slots)                      (mutates k_cache/v_cache)
  kv_append_paged(k, v, k_cache, v_cache, positions, block_table, seat_of_row)   (mutates k_cache/v_cache)
  cp_attn(q, K, V, n_live, softmax_scale) -> out [B, 2048]
  cp_step(q, k, v, K, V, slot, softmax_scale) -> out [B, 2048]         (mutates K/V)

Every op launches on torch.cuda.current_stream() of its tensors' device, so it is recorded by CUDA-graph capture.
The decode workspace is a per-(device, stream) buffer allocated outside capture: run each batch shape once before
capturing (the engine's warm-up passes do, engine/talker.py:120). Its observable content is unchanged by a call (the
ticket counters return to zero), so it is not declared as a mutated argument.
"""
import ctypes
from typing import Optional

import torch

from . import _lib

NH, NKV, HD = 16, 8, 128

_ws = {}                     # (device index, stream handle) -> uint8 workspace tensor


def _paired_rows(k: torch.Tensor, v: torch.Tensor):
    """k and v with one shared row stride, as the kernels take them. The engine often passes k as a fresh tensor (the
    output of RoPE) and v as a strided view of the QKV projection rows (engine/talker.py:159-160,
    engine/code_predictor.py:41-42); then both are made contiguous (one copy each) so the call still works."""
    if k.dim() >= 1 and v.dim() == k.dim() and k.stride() != v.stride():
        return k.contiguous(), v.contiguous()
    return k, v


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(f"q3attn: {msg}")


def _check_cuda_bf16(name: str, t: torch.Tensor) -> None:
    _need(t.is_cuda, f"{name} must be a CUDA tensor (there is no CPU path)")
    _need(t.dtype == torch.bfloat16, f"{name} must be bfloat16, got {t.dtype}")


def workspace(batch: int, num_splits: int, device: torch.device) -> torch.Tensor:
    """The zero-initialised decode workspace for (device, current stream), grown outside capture only."""
    lib = _lib.load()
    with torch.cuda.device(device):
        need = int(lib.q3_paged_decode_workspace_bytes(int(batch), int(num_splits)))
        key = (device.index, _stream(device))
        ws = _ws.get(key)
        if ws is None or ws.numel() < need:
            _need(not torch.cuda.is_current_stream_capturing(),
                  "decode workspace must grow during CUDA-graph capture: run this batch size once before capturing")
            ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=device)
            _ws[key] = ws
        return ws


def _decode_impl(q, k_new, v_new, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, num_splits):
    lib = _lib.load()
    B = q.shape[0]
    _check_cuda_bf16("q", q)
    _check_cuda_bf16("k_cache", k_cache)
    _check_cuda_bf16("v_cache", v_cache)
    _need(q.dim() == 3 and q.shape[1] == NH and q.shape[2] == HD, f"q must be [B, 16, 128], got {tuple(q.shape)}")
    _need(q.stride(2) == 1 and q.stride(1) == HD, "q rows must be contiguous [16, 128]")
    _need(k_cache.dim() == 4 and k_cache.shape[2] == NKV and k_cache.shape[3] == HD and k_cache.is_contiguous()
          and v_cache.shape == k_cache.shape and v_cache.is_contiguous(),
          "k_cache/v_cache must be contiguous [num_pages, page_size, 8, 128]")
    _need(cache_seqlens.dtype == torch.int32 and cache_seqlens.is_cuda and cache_seqlens.numel() == B
          and cache_seqlens.is_contiguous(), "cache_seqlens must be a contiguous int32 CUDA tensor [B]")
    _need(block_table.dtype == torch.int32 and block_table.dim() == 2 and block_table.shape[0] == B
          and block_table.stride(1) == 1, "block_table must be int32 [B, max_pages] with unit inner stride")
    kvs = 0
    if k_new is not None and v_new is not None:
        k_new, v_new = _paired_rows(k_new, v_new)
    if k_new is not None:
        _check_cuda_bf16("k", k_new)
        _check_cuda_bf16("v", v_new)
        _need(k_new.shape == (B, NKV, HD) and v_new.shape == k_new.shape and k_new.stride(2) == 1
              and k_new.stride(1) == HD and v_new.stride() == k_new.stride(), "k/v must be [B, 8, 128] rows")
        kvs = k_new.stride(0)
    out = torch.empty(B, NH, HD, dtype=torch.bfloat16, device=q.device)
    if B == 0:
        return out
    ws = workspace(B, num_splits, q.device)
    with torch.cuda.device(q.device):
        rc = lib.q3_paged_decode(
            q.data_ptr(), q.stride(0), _ptr(k_new), _ptr(v_new), kvs,
            k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0], k_cache.shape[1],
            cache_seqlens.data_ptr(), block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
            B, NH, NKV, HD, float(softmax_scale), out.data_ptr(), out.stride(0),
            ws.data_ptr(), ws.numel(), int(num_splits), _stream(q.device))
    _lib.check(rc, "q3_paged_decode")
    return out


@torch.library.custom_op("q3attn::paged_decode", mutates_args=())
def paged_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cache_seqlens: torch.Tensor,
                 block_table: torch.Tensor, softmax_scale: float, num_splits: int = 0) -> torch.Tensor:
    """Decode attention of q [B,16,128] over cache_seqlens[b] tokens of seat b's pages -> [B,16,128] bf16."""
    return _decode_impl(q, None, None, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, num_splits)


@paged_decode.register_fake
def _(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, num_splits=0):
    return q.new_empty(q.shape[0], NH, HD)


@torch.library.custom_op("q3attn::paged_decode_append", mutates_args=("k_cache", "v_cache"))
def paged_decode_append(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                        v_cache: torch.Tensor, cache_seqlens: torch.Tensor, block_table: torch.Tensor,
                        softmax_scale: float, num_splits: int = 0) -> torch.Tensor:
    """Append k/v [B,8,128] at position cache_seqlens[b], then attend over cache_seqlens[b] + 1 tokens (one launch)."""
    return _decode_impl(q, k, v, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, num_splits)


@paged_decode_append.register_fake
def _(q, k, v, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, num_splits=0):
    return q.new_empty(q.shape[0], NH, HD)


def _norm_rope(q_norm_w, k_norm_w, cos, sin, eps, B):
    """struct q3_qk_norm_rope for [128] bf16 norm weights and cos/sin rows ([B, 128], or [128] / [1, 128] for one row
    shared by every batch row)."""
    for n, t in (("q_norm_w", q_norm_w), ("k_norm_w", k_norm_w), ("cos", cos), ("sin", sin)):
        _check_cuda_bf16(n, t)
        _need(t.shape[-1] == HD and t.stride(-1) == 1, f"{n} must have a contiguous last dim of 128")
    _need(q_norm_w.numel() == HD and k_norm_w.numel() == HD, "norm weights must be [128]")
    c2, s2 = cos.reshape(-1, HD), sin.reshape(-1, HD)
    _need(c2.shape == s2.shape and c2.stride() == s2.stride() and c2.shape[0] in (1, B),
          "cos/sin must both be [B, 128] (one row per batch row) or one [128] row")
    stride = 0 if c2.shape[0] == 1 else c2.stride(0)
    return _lib.QkNormRope(q_norm_w.data_ptr(), k_norm_w.data_ptr(), c2.data_ptr(), s2.data_ptr(), stride, float(eps))


def _qkv_rows(qkv):
    _check_cuda_bf16("qkv", qkv)
    _need(qkv.dim() == 2 and qkv.shape[1] == (NH + 2 * NKV) * HD and qkv.stride(1) == 1,
          "qkv must be [B, 4096] rows: q (16x128) | k (8x128) | v (8x128)")
    return qkv


@torch.library.custom_op("q3attn::paged_decode_qkv", mutates_args=("k_cache", "v_cache"))
def paged_decode_qkv(qkv: torch.Tensor, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, cos: torch.Tensor,
                     sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cache_seqlens: torch.Tensor,
                     block_table: torch.Tensor, softmax_scale: float, eps: float = 1e-6,
                     num_splits: int = 0) -> torch.Tensor:
    """One talker attention layer from the QKV projection (engine/talker.py:69-77): q and k get RMSNorm + RoPE
    (cos/sin row b = position cache_seqlens[b]), k/v are appended at cache_seqlens[b] through the block table, and q
    attends over cache_seqlens[b] + 1 tokens -> [B,16,128] bf16. One launch."""
    lib = _lib.load()
    qkv = _qkv_rows(qkv)
    B = qkv.shape[0]
    _check_cuda_bf16("k_cache", k_cache)
    _check_cuda_bf16("v_cache", v_cache)
    _need(k_cache.dim() == 4 and k_cache.shape[2] == NKV and k_cache.shape[3] == HD and k_cache.is_contiguous()
          and v_cache.shape == k_cache.shape and v_cache.is_contiguous(),
          "k_cache/v_cache must be contiguous [num_pages, page_size, 8, 128]")
    _need(cache_seqlens.dtype == torch.int32 and cache_seqlens.is_cuda and cache_seqlens.numel() == B
          and cache_seqlens.is_contiguous(), "cache_seqlens must be a contiguous int32 CUDA tensor [B]")
    _need(block_table.dtype == torch.int32 and block_table.dim() == 2 and block_table.shape[0] == B
          and block_table.stride(1) == 1, "block_table must be int32 [B, max_pages] with unit inner stride")
    out = torch.empty(B, NH, HD, dtype=torch.bfloat16, device=qkv.device)
    if B == 0:
        return out
    nr = _norm_rope(q_norm_w, k_norm_w, cos, sin, eps, B)
    ws = workspace(B, num_splits, qkv.device)
    with torch.cuda.device(qkv.device):
        rc = lib.q3_paged_decode_qkv(
            qkv.data_ptr(), qkv.stride(0), ctypes.byref(nr), k_cache.data_ptr(), v_cache.data_ptr(),
            k_cache.shape[0], k_cache.shape[1], cache_seqlens.data_ptr(), block_table.data_ptr(),
            block_table.stride(0), block_table.shape[1], B, NH, NKV, HD, float(softmax_scale), out.data_ptr(),
            out.stride(0), ws.data_ptr(), ws.numel(), int(num_splits), _stream(qkv.device))
    _lib.check(rc, "q3_paged_decode_qkv")
    return out


@paged_decode_qkv.register_fake
def _(qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, eps=1e-6,
      num_splits=0):
    return qkv.new_empty(qkv.shape[0], NH, HD)


def _rows(name, t, n_rows_dims=1):
    _check_cuda_bf16(name, t)
    _need(t.dim() >= 2 and t.shape[-1] == HD and t.shape[-2] == NKV and t.stride(-1) == 1 and t.stride(-2) == HD,
          f"{name} must be rows of [8, 128] contiguous elements")
    return t.reshape(-1, NKV, HD) if t.dim() != 3 else t


@torch.library.custom_op("q3attn::kv_append_slots", mutates_args=("k_cache", "v_cache"))
def kv_append_slots(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    slots: torch.Tensor) -> None:
    """k_cache.view(-1,8,128).index_copy_(0, slots, k) and the same for v (engine/talker.py:72-73)."""
    lib = _lib.load()
    k, v = _paired_rows(_rows("k", k), _rows("v", v))
    _check_cuda_bf16("k_cache", k_cache)
    _check_cuda_bf16("v_cache", v_cache)
    _need(k_cache.is_contiguous() and v_cache.is_contiguous() and k_cache.shape == v_cache.shape
          and k_cache.shape[-1] == HD and k_cache.shape[-2] == NKV, "caches must be contiguous [..., 8, 128]")
    _need(v.shape == k.shape and v.stride(0) == k.stride(0), "k and v must have the same shape and row stride")
    s = slots.to(device=k.device, dtype=torch.int64).contiguous()
    _need(s.numel() == k.shape[0], "one slot per row")
    with torch.cuda.device(k.device):
        rc = lib.q3_kv_append_slots(k.data_ptr(), v.data_ptr(), k.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
                                    k_cache.numel() // (NKV * HD), NKV, HD, s.data_ptr(), k.shape[0], _stream(k.device))
    _lib.check(rc, "q3_kv_append_slots")


@torch.library.custom_op("q3attn::kv_append_paged", mutates_args=("k_cache", "v_cache"))
def kv_append_paged(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    positions: torch.Tensor, block_table: torch.Tensor,
                    seat_of_row: Optional[torch.Tensor] = None) -> None:
    """Row i -> token positions[i] of seat seat_of_row[i] (default: seat i) through the block table."""
    lib = _lib.load()
    k, v = _paired_rows(_rows("k", k), _rows("v", v))
    _check_cuda_bf16("k_cache", k_cache)
    _check_cuda_bf16("v_cache", v_cache)
    _need(k_cache.dim() == 4 and k_cache.is_contiguous() and v_cache.is_contiguous() and k_cache.shape == v_cache.shape,
          "caches must be contiguous [num_pages, page_size, 8, 128]")
    _need(v.shape == k.shape and v.stride(0) == k.stride(0), "k and v must have the same shape and row stride")
    pos = positions.to(device=k.device, dtype=torch.int32).contiguous()
    _need(block_table.dtype == torch.int32 and block_table.dim() == 2 and block_table.stride(1) == 1,
          "block_table must be int32 [seats, max_pages]")
    sor = None if seat_of_row is None else seat_of_row.to(device=k.device, dtype=torch.int32).contiguous()
    with torch.cuda.device(k.device):
        rc = lib.q3_kv_append_paged(k.data_ptr(), v.data_ptr(), k.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
                                    k_cache.shape[0], k_cache.shape[1], NKV, HD, pos.data_ptr(), _ptr(sor),
                                    block_table.data_ptr(), block_table.stride(0), block_table.shape[1], k.shape[0],
                                    _stream(k.device))
    _lib.check(rc, "q3_kv_append_paged")


def _rows2d(name, t, cols):
    _check_cuda_bf16(name, t)
    _need(t.dim() == 2 and t.shape[1] == cols and t.stride(1) == 1, f"{name} must be [rows, {cols}] with unit inner stride")


@torch.library.custom_op("q3attn::add_rms_norm", mutates_args=("x",))
def _add_rms_norm_op(x: torch.Tensor, weight: torch.Tensor, residual: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    lib = _lib.load()
    H = x.shape[-1]
    x2 = x.view(-1, H)
    _rows2d("x", x2, H)
    _check_cuda_bf16("weight", weight)
    _need(weight.numel() == H and weight.is_contiguous(), "weight must be [hidden]")
    r2 = None
    if residual is not None:
        r2 = residual.reshape(-1, H)
        _rows2d("residual", r2, H)
        _need(r2.shape[0] == x2.shape[0], "residual must match x")
    out = torch.empty_like(x2)
    with torch.cuda.device(x.device):
        rc = lib.q3_add_rms_norm(x2.data_ptr(), x2.stride(0), _ptr(r2), r2.stride(0) if r2 is not None else 0,
                                 weight.data_ptr(), out.data_ptr(), out.stride(0), x2.shape[0], H, float(eps),
                                 _stream(x.device))
    _lib.check(rc, "q3_add_rms_norm")
    return out.view(x.shape)


@_add_rms_norm_op.register_fake
def _(x, weight, residual, eps):
    return torch.empty_like(x)


def add_rms_norm(x, weight, residual=None, eps: float = 1e-6):
    """RMSNorm (engine/ops.py:51-55) of x [..., H] (H = 1024 or 2048), after x += residual in place when residual is
    given (the residual adds of talker.py:78-79). One launch; returns the normalised rows."""
    return _add_rms_norm_op(x, weight, residual, float(eps))


@torch.library.custom_op("q3attn::silu_mul", mutates_args=())
def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """The MLP gate of engine/ops.py:63-65: silu(g) * u for gate_up = [g | u] [..., 2F] -> [..., F]. One launch."""
    lib = _lib.load()
    F2 = gate_up.shape[-1]
    g2 = gate_up.view(-1, F2)
    _rows2d("gate_up", g2, F2)
    out = torch.empty(g2.shape[0], F2 // 2, dtype=torch.bfloat16, device=gate_up.device)
    with torch.cuda.device(gate_up.device):
        rc = lib.q3_silu_mul(g2.data_ptr(), g2.stride(0), out.data_ptr(), out.stride(0), g2.shape[0], F2 // 2,
                             _stream(gate_up.device))
    _lib.check(rc, "q3_silu_mul")
    return out.view(*gate_up.shape[:-1], F2 // 2)


@silu_mul.register_fake
def _(gate_up):
    return gate_up.new_empty(*gate_up.shape[:-1], gate_up.shape[-1] // 2)


@torch.library.custom_op("q3attn::qk_norm_rope_", mutates_args=("qkv",))
def qk_norm_rope_(qkv: torch.Tensor, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, cos: torch.Tensor,
                  sin: torch.Tensor, eps: float = 1e-6) -> None:
    """q/k RMSNorm + RoPE (engine/ops.py:51-60) in place on QKV rows [T, 4096] (q | k | v): cos/sin [T, 128] (row r
    for row r) or one [128] row. One launch."""
    lib = _lib.load()
    q = _qkv_rows(qkv)
    nr = _norm_rope(q_norm_w, k_norm_w, cos, sin, eps, q.shape[0])
    with torch.cuda.device(qkv.device):
        rc = lib.q3_qk_norm_rope_rows(q.data_ptr(), q.stride(0), ctypes.byref(nr), q.shape[0], _stream(qkv.device))
    _lib.check(rc, "q3_qk_norm_rope_rows")


@torch.library.custom_op("q3attn::ring_window_attn", mutates_args=("k_ring", "v_ring"))
def ring_window_attn(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, k_ring: torch.Tensor,
                     v_ring: torch.Tensor, ring_rows: torch.Tensor, pos: torch.Tensor, past: int, scale: float,
                     write_new: bool = True) -> torch.Tensor:
    """The streaming codec decoder's windowed ring attention for one layer (engine/decoder_stream.py:147-181), fp16.
    q / k_new / v_new [B, n, H, hd] (rotated); k_ring / v_ring [S, RING, H, hd] views of the per-stream rings (e.g.
    K[:, :, layer] of the decoder's [S, RING, L, H, hd] state); ring_rows [B] int64 ring row of each batch entry;
    pos [B] int64 frames decoded before the chunk. With write_new the chunk's K/V go into ring slots (pos + j) % RING.
    Returns [B, n, H * hd] fp16. One launch."""
    lib = _lib.load()
    for name, t in (("q", q), ("k_new", k_new), ("v_new", v_new), ("k_ring", k_ring), ("v_ring", v_ring)):
        _need(t.is_cuda and t.dtype == torch.float16, f"{name} must be a CUDA fp16 tensor")
    _need(q.dim() == 4 and k_new.shape == q.shape and v_new.shape == q.shape and q.stride(3) == 1 and
          q.stride(2) == q.shape[3] and k_new.stride() == q.stride() and v_new.stride() == q.stride(),
          "q / k_new / v_new must be [B, n, H, hd] with equal strides and contiguous heads")
    B, n, H, hd = q.shape
    _need(k_ring.dim() == 4 and k_ring.shape[2:] == (H, hd) and k_ring.stride(3) == 1 and k_ring.stride(2) == hd and
          v_ring.shape == k_ring.shape and v_ring.stride() == k_ring.stride(), "rings must be [S, RING, H, hd] views")
    _need(ring_rows.dtype == torch.int64 and pos.dtype == torch.int64 and ring_rows.numel() == B and
          pos.numel() == B and ring_rows.is_contiguous() and pos.is_contiguous(), "ring_rows / pos: int64 [B]")
    out = torch.empty(B, n, H * hd, dtype=torch.float16, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.q3_ring_window_attn(q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), q.stride(0), q.stride(1),
                                     k_ring.data_ptr(), v_ring.data_ptr(), k_ring.stride(0), k_ring.stride(1),
                                     ring_rows.data_ptr(), pos.data_ptr(), B, n, H, hd, k_ring.shape[1], int(past),
                                     float(scale), int(bool(write_new)), out.data_ptr(), out.stride(0),
                                     out.stride(1), _stream(q.device))
    _lib.check(rc, "q3_ring_window_attn")
    return out


@ring_window_attn.register_fake
def _(q, k_new, v_new, k_ring, v_ring, ring_rows, pos, past, scale, write_new=True):
    return q.new_empty(q.shape[0], q.shape[1], q.shape[2] * q.shape[3])


def pool_pointers(pools) -> torch.Tensor:
    """Device int64 array of the base addresses of per-layer pools (for kv_copy_prefix); build it once, outside
    capture, and keep it with the pools."""
    for t in pools:
        _check_cuda_bf16("pool", t)
        _need(t.is_contiguous() and t.data_ptr() % 16 == 0, "pools must be contiguous and 16-byte aligned")
    return torch.tensor([t.data_ptr() for t in pools], dtype=torch.int64, device=pools[0].device)


def kv_copy_prefix(k_src: torch.Tensor, v_src: torch.Tensor, k_pool_ptrs: torch.Tensor, v_pool_ptrs: torch.Tensor,
                   pool_shape, seat: torch.Tensor, slot: torch.Tensor, block_table: torch.Tensor) -> None:
    """Shared-prefix copy at admission (engine/arrivals.py:139-145 for the prefix rows): for every layer l, batch row
    b and prefix row r, k_src[l, slot[b], r] / v_src[l, slot[b], r] -> position r of seat[b] in layer l's pools
    (k_pool_ptrs / v_pool_ptrs from pool_pointers; pool_shape = (num_pages, page_size, 8, 128)). One launch."""
    lib = _lib.load()
    _check_cuda_bf16("k_src", k_src)
    _check_cuda_bf16("v_src", v_src)
    _need(k_src.dim() == 5 and k_src.shape[3:] == (NKV, HD) and k_src.stride(4) == 1 and k_src.stride(3) == HD and
          k_src.stride(2) == NKV * HD and v_src.shape == k_src.shape and v_src.stride() == k_src.stride(),
          "k_src/v_src must be [layers, slots, k, 8, 128] with contiguous rows")
    L = k_src.shape[0]
    _need(k_pool_ptrs.numel() >= L and v_pool_ptrs.numel() >= L and k_pool_ptrs.dtype == torch.int64,
          "one pool address per layer")
    _need(seat.dtype == torch.int64 and slot.dtype == torch.int64 and seat.numel() == slot.numel(),
          "seat / slot must be int64 [B]")
    _need(block_table.dtype == torch.int32 and block_table.dim() == 2 and block_table.stride(1) == 1,
          "block_table must be int32 [seats, max_pages]")
    num_pages, page = int(pool_shape[0]), int(pool_shape[1])
    with torch.cuda.device(k_src.device):
        rc = lib.q3_kv_copy_prefix(k_src.data_ptr(), v_src.data_ptr(), k_src.stride(0), k_src.stride(1),
                                   k_pool_ptrs.data_ptr(), v_pool_ptrs.data_ptr(), L, num_pages * page, page, NKV, HD,
                                   seat.data_ptr(), slot.data_ptr(), seat.numel(), k_src.shape[2],
                                   block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
                                   _stream(k_src.device))
    _lib.check(rc, "q3_kv_copy_prefix")


def _cp_check(q, K, V):
    _check_cuda_bf16("q", q)
    _check_cuda_bf16("K", K)
    _check_cuda_bf16("V", V)
    B = q.shape[0]
    q2 = q.reshape(B, NH * HD)
    _need(q2.stride(1) == 1, "q rows must be contiguous")
    _need(K.dim() == 4 and K.shape[0] >= B and K.shape[1] == NKV and K.shape[3] == HD and K.stride(3) == 1
          and V.shape == K.shape and V.stride(3) == 1, "K/V must be [B, 8, S, 128] with contiguous 128")
    return q2


@torch.library.custom_op("q3attn::cp_attn", mutates_args=())
def cp_attn_op(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, n_live: int, softmax_scale: float) -> torch.Tensor:
    lib = _lib.load()
    q2 = _cp_check(q, K, V)
    B = q2.shape[0]
    out = torch.empty(B, NH * HD, dtype=torch.bfloat16, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.q3_cp_attn(q2.data_ptr(), q2.stride(0), K.data_ptr(), V.data_ptr(), K.stride(0), K.stride(1),
                            K.stride(2), V.stride(0), V.stride(1), V.stride(2), B, K.shape[2], int(n_live),
                            float(softmax_scale), out.data_ptr(), out.stride(0), _stream(q.device))
    _lib.check(rc, "q3_cp_attn")
    return out


@cp_attn_op.register_fake
def _(q, K, V, n_live, softmax_scale):
    return q.new_empty(q.shape[0], NH * HD)


@torch.library.custom_op("q3attn::cp_step", mutates_args=("K", "V"))
def cp_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, K: torch.Tensor, V: torch.Tensor, slot: int,
            softmax_scale: float) -> torch.Tensor:
    """K[:, :, slot] = k; V[:, :, slot] = v; attention over slots 0..slot -> [B, 2048] (one launch)."""
    lib = _lib.load()
    q2 = _cp_check(q, K, V)
    B = q2.shape[0]
    k3, v3 = _paired_rows(_rows("k", k), _rows("v", v))
    _need(k3.shape[0] == B and v3.shape == k3.shape and v3.stride(0) == k3.stride(0), "k/v must be [B, 8, 128]")
    out = torch.empty(B, NH * HD, dtype=torch.bfloat16, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.q3_cp_step(q2.data_ptr(), q2.stride(0), k3.data_ptr(), v3.data_ptr(), k3.stride(0), K.data_ptr(),
                            V.data_ptr(), K.stride(0), K.stride(1), K.stride(2), V.stride(0), V.stride(1), V.stride(2),
                            B, K.shape[2], int(slot), float(softmax_scale), out.data_ptr(), out.stride(0),
                            _stream(q.device))
    _lib.check(rc, "q3_cp_step")
    return out


@cp_step.register_fake
def _(q, k, v, K, V, slot, softmax_scale):
    return q.new_empty(q.shape[0], NH * HD)


@torch.library.custom_op("q3attn::cp_step_qkv", mutates_args=("K", "V"))
def cp_step_qkv(qkv: torch.Tensor, q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, cos: torch.Tensor,
                sin: torch.Tensor, K: torch.Tensor, V: torch.Tensor, slot: int, softmax_scale: float,
                eps: float = 1e-6) -> torch.Tensor:
    """One code-predictor (step, layer) from the QKV projection (engine/code_predictor.py:40-41, 58, 46-47): q/k
    RMSNorm + RoPE with the cos/sin row of slot p, K/V slot `slot` written, attention over slots 0..slot ->
    [B, 2048]. One launch."""
    lib = _lib.load()
    qkv = _qkv_rows(qkv)
    B = qkv.shape[0]
    _check_cuda_bf16("K", K)
    _check_cuda_bf16("V", V)
    _need(K.dim() == 4 and K.shape[0] >= B and K.shape[1] == NKV and K.shape[3] == HD and K.stride(3) == 1
          and V.shape == K.shape and V.stride(3) == 1, "K/V must be [B, 8, S, 128] with contiguous 128")
    out = torch.empty(B, NH * HD, dtype=torch.bfloat16, device=qkv.device)
    nr = _norm_rope(q_norm_w, k_norm_w, cos, sin, eps, B)
    with torch.cuda.device(qkv.device):
        rc = lib.q3_cp_step_qkv(qkv.data_ptr(), qkv.stride(0), ctypes.byref(nr), K.data_ptr(), V.data_ptr(),
                                K.stride(0), K.stride(1), K.stride(2), V.stride(0), V.stride(1), V.stride(2), B,
                                K.shape[2], int(slot), float(softmax_scale), out.data_ptr(), out.stride(0),
                                _stream(qkv.device))
    _lib.check(rc, "q3_cp_step_qkv")
    return out


@cp_step_qkv.register_fake
def _(qkv, q_norm_w, k_norm_w, cos, sin, K, V, slot, softmax_scale, eps=1e-6):
    return qkv.new_empty(qkv.shape[0], NH * HD)


class SamplerRng:
    """One random stream of q3attn.sample_topk: a seed and a device state [launch index, finish ticket] (int64 x 2)
    that each sampling launch advances by one, CUDA-graph replays included. Draws are Philox4x32-10 of counter
    (row, launch index) under key = seed; they are reproducible from (seed, state) but are not torch's stream."""

    def __init__(self, seed: int, device):
        self.seed = int(seed)
        self.state = torch.zeros(2, dtype=torch.int64, device=device)

    @property
    def launch_index(self) -> int:
        return int(self.state[0])


@torch.library.custom_op("q3attn::sample_topk", mutates_args=("rng_state",))
def _sample_topk_op(logits: torch.Tensor, temperature: float, top_k: int, seed: int, rng_state: torch.Tensor,
                    seen: Optional[torch.Tensor], seat: Optional[torch.Tensor], rep_penalty: float,
                    bias: Optional[torch.Tensor], ngen: Optional[torch.Tensor], min_new: int, eos: int,
                    emb: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    _need(logits.is_cuda and logits.dim() == 2 and logits.stride(1) == 1 and
          logits.dtype in (torch.bfloat16, torch.float32), "logits must be CUDA [B, V] rows, bf16 or fp32")
    B, V = logits.shape
    dev = logits.device
    _need(rng_state.is_cuda and rng_state.dtype == torch.int64 and rng_state.numel() == 2 and
          rng_state.is_contiguous(), "rng_state must be a CUDA int64 [2] tensor (SamplerRng.state)")
    if seen is not None:
        _need(seen.is_cuda and seen.dtype == torch.bool and seen.dim() == 2 and seen.shape[1] == V and
              seen.stride(1) == 1, "seen must be a CUDA bool [S, V] tensor")
    if seen is not None or ngen is not None:
        _need(seat is not None and seat.is_cuda and seat.dtype == torch.int64 and seat.numel() == B and
              seat.is_contiguous(), "seat must be a contiguous CUDA int64 [B] tensor")
    if bias is not None:
        _need(bias.is_cuda and bias.dtype == torch.float32 and bias.numel() == V and bias.is_contiguous(),
              "bias must be a contiguous CUDA fp32 [V] tensor")
    if ngen is not None:
        _need(ngen.is_cuda and ngen.dtype == torch.int64 and ngen.is_contiguous(), "ngen must be CUDA int64")
    ids = torch.empty(B, dtype=torch.int64, device=dev)
    if emb is not None:
        _check_cuda_bf16("emb", emb)
        _need(emb.dim() == 2 and emb.stride(1) == 1 and emb.shape[0] >= V and emb.shape[1] % 4 == 0,
              "emb must be a [rows >= V, dim] bf16 table with dim a multiple of 4")
        emb_out = torch.empty(B, emb.shape[1], dtype=torch.bfloat16, device=dev)
    else:
        emb_out = torch.empty(0, dtype=torch.bfloat16, device=dev)
    p = _lib.Sampler(logits.data_ptr(), 0 if logits.dtype == torch.bfloat16 else 1, logits.stride(0), B, V,
                     int(top_k), float(temperature), _ptr(seen), seen.stride(0) if seen is not None else 0,
                     _ptr(seat), float(rep_penalty), _ptr(bias), _ptr(ngen), int(min_new), int(eos),
                     int(seed) & 0xFFFFFFFFFFFFFFFF, rng_state.data_ptr(), ids.data_ptr(), 1, _ptr(emb),
                     emb.stride(0) if emb is not None else 0, emb.shape[1] if emb is not None else 0,
                     emb_out.data_ptr() if emb is not None else None, emb_out.stride(0) if emb is not None else 0)
    with torch.cuda.device(dev):
        rc = lib.q3_sample_topk(ctypes.byref(p), _stream(dev))
    _lib.check(rc, "q3_sample_topk")
    return ids, emb_out


@_sample_topk_op.register_fake
def _(logits, temperature, top_k, seed, rng_state, seen, seat, rep_penalty, bias, ngen, min_new, eos, emb):
    B = logits.shape[0]
    e = logits.new_empty(B, emb.shape[1], dtype=torch.bfloat16) if emb is not None else \
        logits.new_empty(0, dtype=torch.bfloat16)
    return logits.new_empty(B, dtype=torch.int64), e


def sample_topk(logits, temperature: float, k: int, rng: SamplerRng, *, seen=None, seat=None, rep_penalty=1.0,
                bias=None, ngen=None, min_new=0, eos=-1, emb=None):
    """engine/ops.py:68-76 (top-k, softmax(vals / temperature), one draw) on the GPU, with the optional logit
    processing of engine/talker.py:91-94 applied first (repetition penalty over seen[seat[b]], + bias, EOS masked while
    ngen[seat[b]] < min_new) and the optional embedding lookup of the sampled ids after. logits [B, V] bf16 or fp32
    (V <= 4096, k <= 64). Returns ids [B] int64, or (ids, emb[ids]) when emb is given. One launch."""
    ids, e = _sample_topk_op(logits, float(temperature), int(k), rng.seed, rng.state, seen, seat, float(rep_penalty),
                             bias, ngen, int(min_new), int(eos), emb)
    return (ids, e) if emb is not None else ids


def _prefill_impl(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale, causal, k_cache=None,
                  v_cache=None, prefix_lens=None, seat_ids=None, block_table=None, write_kv=False):
    lib = _lib.load()
    _check_cuda_bf16("q", q)
    _check_cuda_bf16("k", k)
    _check_cuda_bf16("v", v)
    k, v = _paired_rows(k, v)
    _need(q.dim() == 3 and q.shape[1] == NH and q.shape[2] == HD and q.stride(2) == 1 and q.stride(1) == HD,
          "q must be packed rows [T, 16, 128]")
    _need(k.dim() == 3 and k.shape[1] == NKV and k.shape[2] == HD and k.stride(2) == 1 and k.stride(1) == HD
          and v.shape == k.shape and v.stride() == k.stride(), "k/v must be packed rows [T, 8, 128] with equal strides")
    for name, t in (("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_k", cu_seqlens_k)):
        _need(t.dtype == torch.int32 and t.is_cuda and t.dim() == 1 and t.is_contiguous(), f"{name}: contiguous int32")
    n = cu_seqlens_q.numel() - 1
    _need(cu_seqlens_k.numel() == n + 1, "cu_seqlens_q and cu_seqlens_k describe different sequence counts")
    out = torch.empty(q.shape[0], NH, HD, dtype=torch.bfloat16, device=q.device)
    paged = k_cache is not None
    if paged:
        _check_cuda_bf16("k_cache", k_cache)
        _check_cuda_bf16("v_cache", v_cache)
        _need(k_cache.dim() == 4 and k_cache.is_contiguous() and v_cache.shape == k_cache.shape and v_cache.is_contiguous(),
              "caches must be contiguous [num_pages, page_size, 8, 128]")
        _need(block_table is not None and block_table.dtype == torch.int32 and block_table.stride(1) == 1,
              "block_table must be int32 [seats, max_pages]")
    pl = None if prefix_lens is None else prefix_lens.to(device=q.device, dtype=torch.int32).contiguous()
    si = None if seat_ids is None else seat_ids.to(device=q.device, dtype=torch.int32).contiguous()
    if n == 0 or q.shape[0] == 0:
        return out
    with torch.cuda.device(q.device):
        rc = lib.q3_prefill(
            q.data_ptr(), q.stride(0), q.shape[0], k.data_ptr(), v.data_ptr(), k.stride(0), k.shape[0],
            cu_seqlens_q.data_ptr(),
            cu_seqlens_k.data_ptr(), n, int(max_seqlen_q), _ptr(pl), _ptr(si),
            _ptr(k_cache) if paged else None, _ptr(v_cache) if paged else None,
            k_cache.shape[0] if paged else 0, k_cache.shape[1] if paged else 0,
            _ptr(block_table) if paged else None, block_table.stride(0) if paged else 0,
            block_table.shape[1] if paged else 0, int(bool(write_kv)), int(bool(causal)), NH, NKV, HD,
            float(softmax_scale), out.data_ptr(), out.stride(0), _stream(q.device))
    _lib.check(rc, "q3_prefill")
    return out


@torch.library.custom_op("q3attn::prefill", mutates_args=())
def prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
            max_seqlen_q: int, softmax_scale: float, causal: bool = True) -> torch.Tensor:
    """Packed varlen prefill attention: q rows [T, 16, 128] of each sequence over its k/v rows [T', 8, 128]
    (N_i >= R_i keys, causal aligned to the bottom right) -> [T, 16, 128] bf16."""
    return _prefill_impl(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale, causal)


@prefill.register_fake
def _(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale, causal=True):
    return q.new_empty(q.shape[0], NH, HD)


@torch.library.custom_op("q3attn::prefill_paged", mutates_args=("k_cache", "v_cache"))
def prefill_paged(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor, max_seqlen_q: int, prefix_lens: torch.Tensor,
                  seat_ids: torch.Tensor, block_table: torch.Tensor, softmax_scale: float, causal: bool = True,
                  write_kv: bool = True) -> torch.Tensor:
    """Chunked prefill into pages: sequence i's new k/v rows go to positions prefix_lens[i].. of seat seat_ids[i]
    (write_kv) and its queries attend over the cached prefix (read through the block table) plus the new rows."""
    return _prefill_impl(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale, causal, k_cache, v_cache,
                         prefix_lens, seat_ids, block_table, write_kv)


@prefill_paged.register_fake
def _(q, k, v, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, prefix_lens, seat_ids, block_table,
      softmax_scale, causal=True, write_kv=True):
    return q.new_empty(q.shape[0], NH, HD)


def set_ring_frame_kernel(kernel: int) -> int:
    """Select the one-frame ring attention kernel. 6 (default): nothing staged, 4 (head_dim 64) or 8 (128) warps per
    (stream, head) loading their rows straight into registers (past <= 79; other calls run 2); 2: scalar math, one warp per head,
    4 x 64 or 2 x 128 heads per CTA; 1: scalar math, one CTA per (stream, head); 0 / 3 / 4: tensor cores, one warp per
    head, 4 / 2 / 1 heads of 64 (2 / 1 / 1 of 128) per CTA; 5: persistent TMA pipeline, quads of four warps per
    (stream, head) fed by producer warps (head_dim 64). Calls a selection does not fit run 1. Returns the previous
    selection."""
    return int(_lib.load().q3_set_ring_frame_kernel(int(kernel)))


def set_ring_chunk_kernel(kernel: int) -> int:
    """Select the ring attention kernel for chunks of 2 .. 17 frames. 1 (default): one CTA per (stream, head), tensor
    cores, also for every call another selection does not fit; 0 / 2 / 3: tensor cores, one warp per head, 2 / 4 / 1
    heads of 64 (1 / 2 / 1 of 128) per CTA, up to 16 frames; 4: the persistent TMA pipeline (2 .. 8 frames, head_dim
    64). Returns the previous selection."""
    return int(_lib.load().q3_set_ring_chunk_kernel(int(kernel)))


def set_prefill_kernel(kernel: int) -> int:
    """Select the prefill kernel (0: the warp-specialised TMA kernel where the call fits it, else the single-warpgroup
    kernel; 1: the single-warpgroup kernel always). Returns the previous selection."""
    return int(_lib.load().q3_set_prefill_kernel(int(kernel)))


def set_decode_variant(variant: int) -> int:
    """Select the decode kernel variant (0: 8-token chunks x 3 stages, two CTAs/SM; 1: 16-token x 3, one CTA/SM;
    2: 8-token x 2, two CTAs/SM; 3 / 4: warp-MMA scoring with early stage release, 8-token x 3 / 2, two CTAs/SM;
    5 (default): dedicated producer warps, one CTA/SM running two 8-token x 3 chunk streams)."""
    _ws.clear()
    return int(_lib.load().q3_set_decode_variant(int(variant)))
