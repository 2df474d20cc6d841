"""ctypes binding of libq3attn.so (the C ABI declared in include/q3attn.h).

The library is loaded from this package directory. There is no fallback: if it is missing or fails to load, importing
the ops raises, so a caller can never silently run something other than the CUDA kernels.
"""
import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libq3attn.so")

Q3_OK, Q3_ERR_INVALID, Q3_ERR_UNSUPPORTED, Q3_ERR_ALIGNMENT, Q3_ERR_WORKSPACE, Q3_ERR_CUDA, Q3_ERR_SCRATCH_LIMIT = range(7)
STATUS_WAIT_TIMEOUT, STATUS_BAD_PAGE, STATUS_BAD_LENGTH = 1, 2, 4

_P, _I32, _I64, _F32, _SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t


class QkNormRope(ctypes.Structure):
    """struct q3_qk_norm_rope (include/q3attn.h): q/k RMSNorm weights and RoPE rows fused into the attention kernels."""
    _fields_ = [("q_norm_weight", _P), ("k_norm_weight", _P), ("cos", _P), ("sin", _P),
                ("rope_row_stride", _I64), ("eps", _F32)]


_NR = ctypes.POINTER(QkNormRope)


class Sampler(ctypes.Structure):
    """struct q3_sampler (include/q3attn.h): logit processing + top-k sampling of one batch of rows."""
    _fields_ = [("logits", _P), ("logits_dtype", _I32), ("row_stride", _I64), ("batch", _I32), ("vocab", _I32),
                ("top_k", _I32), ("temperature", _F32), ("seen", _P), ("seen_row_stride", _I64), ("seat", _P),
                ("repetition_penalty", _F32), ("bias", _P), ("ngen", _P), ("min_new", _I32), ("eos_id", _I32),
                ("seed", ctypes.c_uint64), ("rng_state", _P), ("out_ids", _P), ("out_stride", _I64), ("emb", _P),
                ("emb_row_stride", _I64), ("emb_dim", _I32), ("emb_out", _P), ("emb_out_row_stride", _I64)]

# name -> (restype, argtypes); every symbol include/q3attn.h declares
SIGNATURES = {
    "q3_version": (ctypes.c_int, []),
    "q3_error_string": (ctypes.c_char_p, [ctypes.c_int]),
    "q3_last_cuda_error": (ctypes.c_char_p, []),
    "q3_device_sm_count": (ctypes.c_int, []),
    "q3_read_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]),
    "q3_paged_decode_workspace_bytes": (_SZ, [_I32, _I32]),
    "q3_paged_decode": (ctypes.c_int, [_P, _I64, _P, _P, _I64, _P, _P, _I32, _I32, _P, _P, _I64, _I32,
                                       _I32, _I32, _I32, _I32, _F32, _P, _I64, _P, _SZ, _I32, _P]),
    "q3_paged_decode_noalloc": (ctypes.c_int, [_P, _I64, _P, _P, _I64, _P, _P, _I32, _I32, _P, _P, _I64, _I32,
                                               _I32, _I32, _I32, _I32, _F32, _P, _I64, _I32, _P]),
    "q3_paged_decode_qkv": (ctypes.c_int, [_P, _I64, _NR, _P, _P, _I32, _I32, _P, _P, _I64, _I32,
                                           _I32, _I32, _I32, _I32, _F32, _P, _I64, _P, _SZ, _I32, _P]),
    "q3_set_decode_variant": (ctypes.c_int, [ctypes.c_int]),
    "q3_paged_decode_resident_ctas": (ctypes.c_int, [ctypes.c_int]),
    "q3_set_prefill_kernel": (ctypes.c_int, [ctypes.c_int]),
    "q3_prefill": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _I32, _I32, _P, _P, _P, _P, _I32, _I32, _P, _I64,
                                  _I32, _I32, _I32, _I32, _I32, _I32, _F32, _P, _I64, _P]),
    "q3_kv_append_slots": (ctypes.c_int, [_P, _P, _I64, _P, _P, _I64, _I32, _I32, _P, _I32, _P]),
    "q3_kv_append_paged": (ctypes.c_int, [_P, _P, _I64, _P, _P, _I32, _I32, _I32, _I32, _P, _P, _P, _I64, _I32,
                                          _I32, _P]),
    "q3_cp_attn": (ctypes.c_int, [_P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _I32, _I32, _F32,
                                  _P, _I64, _P]),
    "q3_cp_step": (ctypes.c_int, [_P, _I64, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _I32,
                                  _I32, _F32, _P, _I64, _P]),
    "q3_sample_topk": (ctypes.c_int, [ctypes.POINTER(Sampler), _P]),
    "q3_add_rms_norm": (ctypes.c_int, [_P, _I64, _P, _I64, _P, _P, _I64, _I64, _I32, _F32, _P]),
    "q3_silu_mul": (ctypes.c_int, [_P, _I64, _P, _I64, _I64, _I32, _P]),
    "q3_qk_norm_rope_rows": (ctypes.c_int, [_P, _I64, _NR, _I64, _P]),
    "q3_set_ring_frame_kernel": (ctypes.c_int, [ctypes.c_int]),
    "q3_set_ring_chunk_kernel": (ctypes.c_int, [ctypes.c_int]),
    "q3_selftest_bounded_wait": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_void_p]),
    "q3_ring_window_attn": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _P, _P, _I64, _I64, _P, _P, _I32, _I32, _I32,
                                           _I32, _I32, _I32, _F32, _I32, _P, _I64, _I64, _P]),
    "q3_kv_copy_prefix": (ctypes.c_int, [_P, _P, _I64, _I64, _P, _P, _I32, _I64, _I32, _I32, _I32, _P, _P, _I32, _I32,
                                         _P, _I64, _I32, _P]),
    "q3_cp_step_qkv": (ctypes.c_int, [_P, _I64, _NR, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I32, _I32,
                                      _I32, _F32, _P, _I64, _P]),
}

_lib = None


class Q3Error(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises Q3Error if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise Q3Error(f"q3attn CUDA library not built ({LIB_PATH} missing): run `python -m q3attn.build` "
                      "from qwen3-tts-engine_b200/ or __graft_entry__.build()")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != Q3_OK:
        lib = load()
        msg = lib.q3_error_string(rc).decode()
        if rc == Q3_ERR_CUDA:
            msg += f" ({lib.q3_last_cuda_error().decode()})"
        raise Q3Error(f"{what}: {msg}")


def read_status(clear: bool = True) -> int:
    """Device status bits (STATUS_*) raised by kernels since the last clear, for the current device."""
    v = ctypes.c_uint32(0)
    check(load().q3_read_status(ctypes.byref(v), int(clear)), "q3_read_status")
    return int(v.value)
