"""Drop-in entry points with the reference engine's call signatures, backed by the q3attn kernels.

The engine imports ``flash_attn_with_kvcache, flash_attn_varlen_func`` (engine/talker.py:13) and ``flash_attn_func``
(engine/arrivals.py:30) from flash-attn. These functions accept the same arguments for the shapes the engine uses
(GQA 16/8, head_dim 128, bf16) and raise NotImplementedError for flash-attn features the engine never passes (sliding
windows, softcap, ALiBi, rotary inside the kernel, cache_batch_idx/leftpad, returning the LSE), rather than computing
something else. ``cp_attn`` keeps the signature of engine/cp_attn.py:33, and ``cp_step`` is the code predictor's slot
write + attention (engine/code_predictor.py:58, 46-47) as one call.
"""
import torch

from . import ops

NH, NKV, HD = ops.NH, ops.NKV, ops.HD


def _unsupported(**kw):
    bad = [k for k, v in kw.items() if v]
    if bad:
        raise NotImplementedError(f"q3attn does not implement flash-attn option(s) {bad}")


def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, rotary_cos=None, rotary_sin=None, cache_seqlens=None,
                            cache_batch_idx=None, cache_leftpad=None, block_table=None, softmax_scale=None,
                            causal=False, window_size=(-1, -1), softcap=0.0, rotary_interleaved=True,
                            alibi_slopes=None, num_splits=0, return_softmax_lse=False):
    """Decode attention over a (paged) KV cache, the call at engine/talker.py:77.

    q [B, 1, 16, 128]; k_cache/v_cache [num_pages, page_size, 8, 128] with block_table int32 [B, max_pages], or
    [B, seqlen_max, 8, 128] without one; cache_seqlens int32 [B] (or an int). With k/v [B, 1, 8, 128] the new rows are
    appended at cache_seqlens[b] first and attended too (one fused launch). Returns [B, 1, 16, 128] bf16."""
    _unsupported(rotary_cos=rotary_cos is not None, rotary_sin=rotary_sin is not None,
                 cache_batch_idx=cache_batch_idx is not None, cache_leftpad=cache_leftpad is not None,
                 window_size=tuple(window_size) != (-1, -1), softcap=softcap != 0.0, alibi_slopes=alibi_slopes is not None,
                 return_softmax_lse=return_softmax_lse)
    B = q.shape[0]
    if q.dim() != 4 or q.shape[1] != 1:
        raise NotImplementedError("q3attn decode takes one query token per sequence (q [B, 1, 16, 128])")
    q3 = q.view(B, NH, HD) if q.is_contiguous() else q[:, 0]
    if block_table is None:                      # contiguous cache: seat b owns "page" b of size seqlen_max
        block_table = torch.arange(B, dtype=torch.int32, device=q.device)[:, None]
    if cache_seqlens is None:
        raise NotImplementedError("cache_seqlens is required")
    if isinstance(cache_seqlens, int):
        cache_seqlens = torch.full((B,), cache_seqlens, dtype=torch.int32, device=q.device)
    scale = float(softmax_scale) if softmax_scale is not None else HD ** -0.5
    if k is not None:
        if v is None or k.shape[1] != 1:
            raise NotImplementedError("k/v append takes one new token per sequence ([B, 1, 8, 128])")
        out = ops.paged_decode_append(q3, k[:, 0], v[:, 0], k_cache, v_cache, cache_seqlens, block_table, scale,
                                      int(num_splits))
    else:
        out = ops.paged_decode(q3, k_cache, v_cache, cache_seqlens, block_table, scale, int(num_splits))
    return out.view(B, 1, NH, HD)


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, dropout_p=0.0,
                           softmax_scale=None, causal=False, window_size=(-1, -1), softcap=0.0, alibi_slopes=None,
                           deterministic=False, return_attn_probs=False, block_table=None):
    """Packed varlen attention, the call at engine/talker.py:169. q [Tq,16,128], k/v [Tk,8,128], cu_seqlens int32;
    causal masks are aligned to the bottom right (flash-attention's convention). Returns [Tq, 16, 128] bf16."""
    _unsupported(dropout_p=dropout_p != 0.0, window_size=tuple(window_size) != (-1, -1), softcap=softcap != 0.0,
                 alibi_slopes=alibi_slopes is not None, return_attn_probs=return_attn_probs,
                 block_table=block_table is not None)
    scale = float(softmax_scale) if softmax_scale is not None else HD ** -0.5
    return ops.prefill(q, k, v, cu_seqlens_q, cu_seqlens_k, int(max_seqlen_q), scale, bool(causal))


def flash_attn_func(q, k, v, dropout_p=0.0, softmax_scale=None, causal=False, window_size=(-1, -1), softcap=0.0,
                    alibi_slopes=None, deterministic=False, return_attn_probs=False):
    """Batched attention, the call at engine/arrivals.py:148: q [S,R,16,128] over k/v [S,n,8,128] (n >= R), causal
    aligned to the bottom right (query i sees the n-R prefix keys and the new keys <= i). Returns [S, R, 16, 128]."""
    _unsupported(dropout_p=dropout_p != 0.0, window_size=tuple(window_size) != (-1, -1), softcap=softcap != 0.0,
                 alibi_slopes=alibi_slopes is not None, return_attn_probs=return_attn_probs)
    S, R = q.shape[0], q.shape[1]
    n = k.shape[1]
    dev = q.device
    cu_q = torch.arange(S + 1, dtype=torch.int32, device=dev) * R
    cu_k = torch.arange(S + 1, dtype=torch.int32, device=dev) * n
    scale = float(softmax_scale) if softmax_scale is not None else HD ** -0.5
    o = ops.prefill(q.reshape(S * R, NH, HD), k.reshape(S * n, NKV, HD), v.reshape(S * n, NKV, HD), cu_q, cu_k, R,
                    scale, bool(causal))
    return o.view(S, R, NH, HD)


def cp_attn(q, K, V, n_live, scale):
    """``cp_attn(q, K, V, n_live, scale) -> o [B, 2048]`` (engine/cp_attn.py:33-39): q [B,16,128] or [B,2048]; K/V
    [B,8,16,128] whose batch stride may exceed the live batch; slots 0..n_live-1 attended; fp32 scores, softmax,
    probabilities and P.V; bf16 output."""
    return ops.cp_attn_op(q, K, V, int(n_live), float(scale))


def cp_step(q, k, v, K, V, p, scale):
    """``K[:, :, p] = k; V[:, :, p] = v`` (engine/code_predictor.py:58) then the attention of code_predictor.py:46-47
    over slots 0..p, in one launch -> [B, 2048]."""
    return ops.cp_step(q, k, v, K, V, int(p), float(scale))
