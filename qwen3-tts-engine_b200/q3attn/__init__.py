"""q3attn: B200 (sm_100a) attention hot path of the Qwen3-TTS streaming engine, behind a C ABI (include/q3attn.h).

Public Python surface (drop-ins for the engine's imports):
  flash_attn_with_kvcache  (engine/talker.py:13, 77)       paged decode attention, optional fused K/V append
  cp_attn / cp_step        (engine/cp_attn.py:33)          code-predictor attention, optional fused slot append
  ops.kv_append_slots / kv_append_paged                    the engine's index_copy_ appends into the page pool
The CUDA library is required: nothing here computes attention on the CPU.
"""
from . import _lib, ops  # noqa: F401
from .flash_api import cp_attn, cp_step, flash_attn_func, flash_attn_varlen_func, flash_attn_with_kvcache  # noqa: F401
from .ops import (SamplerRng, add_rms_norm, cp_step_qkv, kv_append_paged, kv_append_slots,  # noqa: F401
                  paged_decode, paged_decode_append, paged_decode_qkv, prefill, prefill_paged, qk_norm_rope_,
                  ring_window_attn, sample_topk, set_decode_variant, set_prefill_kernel, set_ring_chunk_kernel,
                  set_ring_frame_kernel, silu_mul)

__version__ = "0.1.0"
