"""CPU: the C-ABI library loads, exports every symbol include/q3attn.h declares, and rejects bad arguments on the host
(no kernel is launched: every case below fails its argument check before any CUDA call)."""
import ctypes
import os
import re

import pytest
import torch

from q3attn import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(REPO, "include", "q3attn.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(q3_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = header_functions()
    assert len(names) >= 11
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/q3attn.h but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature in q3attn._lib"


def test_version_and_error_strings():
    lib = _lib.load()
    assert lib.q3_version() >= 100
    for code in range(6):
        assert lib.q3_error_string(code)
    assert b"unsupported" in lib.q3_error_string(_lib.Q3_ERR_UNSUPPORTED)


def test_decode_rejects_unsupported_family_before_cuda():
    lib = _lib.load()
    rc = lib.q3_paged_decode(1, 4096, None, None, 0, 1, 1, 10, 16, 1, 1, 4, 4, 4, 32, 8, 128, 0.1, 1, 4096, 1, 1 << 20,
                             0, None)
    assert rc == _lib.Q3_ERR_UNSUPPORTED
    rc = lib.q3_paged_decode(1, 4096, None, None, 0, 1, 1, 10, 16, 1, 1, 4, 4, 4, 16, 8, 64, 0.1, 1, 4096, 1, 1 << 20,
                             0, None)
    assert rc == _lib.Q3_ERR_UNSUPPORTED


def test_decode_rejects_invalid_sizes_before_cuda():
    lib = _lib.load()
    # negative batch, zero pages, zero page size, k without v
    assert lib.q3_paged_decode(1, 2048, None, None, 0, 1, 1, 10, 16, 1, 1, 4, 4, -1, 16, 8, 128, 0.1, 1, 2048, 1, 1,
                               0, None) == _lib.Q3_ERR_INVALID
    assert lib.q3_paged_decode(1, 2048, None, None, 0, 1, 1, 0, 16, 1, 1, 4, 4, 2, 16, 8, 128, 0.1, 1, 2048, 1, 1, 0,
                               None) == _lib.Q3_ERR_INVALID
    assert lib.q3_paged_decode(1, 2048, 16, None, 1024, 1, 1, 10, 16, 1, 1, 4, 4, 2, 16, 8, 128, 0.1, 1, 2048, 1, 1,
                               0, None) == _lib.Q3_ERR_INVALID
    # block-table stride shorter than the pages it claims
    assert lib.q3_paged_decode(1, 2048, None, None, 0, 1, 1, 10, 16, 1, 1, 2, 4, 2, 16, 8, 128, 0.1, 1, 2048, 1, 1,
                               0, None) == _lib.Q3_ERR_INVALID
    # batch 0 is a no-op
    assert lib.q3_paged_decode(None, 2048, None, None, 0, None, None, 10, 16, None, None, 4, 4, 0, 16, 8, 128, 0.1,
                               None, 2048, None, 0, 0, None) == _lib.Q3_OK


def test_decode_rejects_misaligned_pools_before_cuda():
    lib = _lib.load()
    assert lib.q3_paged_decode(16, 2048, None, None, 0, 24, 32, 10, 16, 64, 64, 4, 4, 2, 16, 8, 128, 0.1, 16, 2048, 256,
                               1 << 20, 0, None) == _lib.Q3_ERR_ALIGNMENT


def test_cp_rejects_bad_slot_counts_before_cuda():
    lib = _lib.load()
    args = (16, 2048, 16, 16, 16384, 2048, 128, 16384, 2048, 128)
    assert lib.q3_cp_attn(*args, 4, 16, 0, 0.1, 16, 2048, None) == _lib.Q3_ERR_INVALID      # n_live 0
    assert lib.q3_cp_attn(*args, 4, 16, 17, 0.1, 16, 2048, None) == _lib.Q3_ERR_INVALID     # n_live > slots
    assert lib.q3_cp_attn(*args, 4, 32, 17, 0.1, 16, 2048, None) == _lib.Q3_ERR_UNSUPPORTED  # > 16 slots attended
    assert lib.q3_cp_attn(*args, 0, 16, 3, 0.1, 16, 2048, None) == _lib.Q3_OK               # empty batch


def _norm_rope(qn=256, kn=512, cos=768, sin=1024, stride=128, eps=1e-6):
    return _lib.QkNormRope(qn, kn, cos, sin, stride, eps)


def _decode_qkv(nr, qkv=4096, stride=4096, batch=2):
    lib = _lib.load()
    return lib.q3_paged_decode_qkv(qkv, stride, nr, 8192, 8192 * 4, 10, 16, 64, 64, 4, 4, batch, 16, 8, 128, 0.1,
                                   8192 * 8, 2048, 8192 * 16, 1 << 20, 0, None)


def test_fused_decode_rejects_bad_norm_rope_before_cuda():
    assert _decode_qkv(None) == _lib.Q3_ERR_INVALID                                        # no norm/rope struct
    nr = _norm_rope()
    assert _decode_qkv(ctypes.byref(nr), stride=2048) == _lib.Q3_ERR_INVALID               # row shorter than q|k|v
    nr = _norm_rope(kn=None)
    assert _decode_qkv(ctypes.byref(nr)) == _lib.Q3_ERR_INVALID                            # missing k weight
    nr = _norm_rope(stride=-128)
    assert _decode_qkv(ctypes.byref(nr)) == _lib.Q3_ERR_INVALID                            # negative rope stride
    nr = _norm_rope(cos=770)
    assert _decode_qkv(ctypes.byref(nr)) == _lib.Q3_ERR_ALIGNMENT                          # cos row not 8-byte aligned
    nr = _norm_rope()
    assert _decode_qkv(ctypes.byref(nr), batch=0) == _lib.Q3_OK                           # empty batch is a no-op


def test_fused_cp_step_rejects_bad_norm_rope_before_cuda():
    lib = _lib.load()
    strides = (16384, 2048, 128, 16384, 2048, 128)
    assert lib.q3_cp_step_qkv(4096, 4096, None, 8192, 8192, *strides, 4, 16, 2, 0.1, 8192, 2048, None) == \
        _lib.Q3_ERR_INVALID
    nr = _norm_rope()
    assert lib.q3_cp_step_qkv(4096, 2048, ctypes.byref(nr), 8192, 8192, *strides, 4, 16, 2, 0.1, 8192, 2048,
                              None) == _lib.Q3_ERR_INVALID                                  # row shorter than q|k|v
    assert lib.q3_cp_step_qkv(4096, 4096, ctypes.byref(nr), 8192, 8192, *strides, 4, 16, 16, 0.1, 8192, 2048,
                              None) == _lib.Q3_ERR_INVALID                                  # slot 16 of 16
    nr = _norm_rope(sin=1030)
    assert lib.q3_cp_step_qkv(4096, 4096, ctypes.byref(nr), 8192, 8192, *strides, 4, 16, 2, 0.1, 8192, 2048,
                              None) == _lib.Q3_ERR_ALIGNMENT


def test_append_rejects_bad_arguments_before_cuda():
    lib = _lib.load()
    assert lib.q3_kv_append_slots(16, 16, 1024, 16, 16, 0, 8, 128, 16, 4, None) == _lib.Q3_ERR_INVALID   # no pool
    assert lib.q3_kv_append_slots(16, 16, 1000, 16, 16, 64, 8, 128, 16, 4, None) == _lib.Q3_ERR_INVALID  # stride < row
    assert lib.q3_kv_append_slots(24, 16, 1024, 16, 16, 64, 8, 128, 16, 4, None) == _lib.Q3_ERR_ALIGNMENT
    assert lib.q3_kv_append_paged(16, 16, 1024, 16, 16, 4, 16, 8, 128, 16, None, 16, 2, 4, 3, None) == \
        _lib.Q3_ERR_INVALID                                                                             # bt stride < pages


def test_ops_refuse_cpu_tensors():
    import q3attn
    q = torch.zeros(2, 16, 128, dtype=torch.bfloat16)
    kc = torch.zeros(4, 16, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        q3attn.paged_decode(q, kc, kc, torch.ones(2, dtype=torch.int32), torch.zeros(2, 2, dtype=torch.int32), 0.1, 0)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        q3attn.cp_attn(q, torch.zeros(2, 8, 16, 128, dtype=torch.bfloat16), torch.zeros(2, 8, 16, 128,
                                                                                          dtype=torch.bfloat16), 3, 0.1)


def test_flash_api_refuses_unimplemented_options():
    import q3attn
    q = torch.zeros(2, 1, 16, 128, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        q3attn.flash_attn_with_kvcache(q, q, q, cache_seqlens=1, window_size=(4, 0))
    with pytest.raises(NotImplementedError):
        q3attn.flash_attn_with_kvcache(q, q, q, cache_seqlens=1, return_softmax_lse=True)


def _ring(q=16, batch=2, n=1, heads=4, hd=64, ring=88, past=71, qkv_bs=1024, qkv_fs=256, slot_s=256, out=16,
          ring_rows=64, pos=64):
    lib = _lib.load()
    return lib.q3_ring_window_attn(q, q, q, qkv_bs, qkv_fs, 32, 48, 88 * 256, slot_s, ring_rows, pos, batch, n,
                                   heads, hd, ring, past, 0.125, 0, out, qkv_bs, qkv_fs, None)


def test_ring_rejects_bad_arguments_before_cuda():
    assert _ring(batch=-1) == _lib.Q3_ERR_INVALID
    assert _ring(hd=96) == _lib.Q3_ERR_UNSUPPORTED                       # head_dim 64 or 128 only
    assert _ring(ring=129) == _lib.Q3_ERR_UNSUPPORTED                    # ring <= 128 slots
    assert _ring(n=18, ring=120, past=71) == _lib.Q3_ERR_UNSUPPORTED     # chunk <= 17 frames
    assert _ring(n=18, ring=88, past=71) == _lib.Q3_ERR_UNSUPPORTED
    assert _ring(n=17, ring=88, past=72) == _lib.Q3_ERR_INVALID          # chunk slots must lie outside every window
    assert _ring(ring_rows=None) == _lib.Q3_ERR_INVALID
    assert _ring(qkv_fs=128) == _lib.Q3_ERR_INVALID                      # frame stride shorter than heads x head_dim
    assert _ring(q=24) == _lib.Q3_ERR_ALIGNMENT                          # q not 16-byte aligned
    assert _ring(batch=0) == _lib.Q3_OK and _ring(n=0) == _lib.Q3_OK     # empty calls are no-ops


def _sampler(**kw):
    f = dict(logits=64, logits_dtype=0, row_stride=3072, batch=4, vocab=3072, top_k=50, temperature=0.9, seen=None,
             seen_row_stride=0, seat=None, repetition_penalty=1.0, bias=None, ngen=None, min_new=0, eos_id=0, seed=1,
             rng_state=128, out_ids=256, out_stride=1, emb=None, emb_row_stride=0, emb_dim=0, emb_out=None,
             emb_out_row_stride=0)
    f.update(kw)
    s = _lib.Sampler(**f)
    return _lib.load().q3_sample_topk(ctypes.byref(s), None)


def test_sampler_rejects_bad_arguments_before_cuda():
    assert _lib.load().q3_sample_topk(None, None) == _lib.Q3_ERR_INVALID
    assert _sampler(vocab=5000, row_stride=5000) == _lib.Q3_ERR_UNSUPPORTED        # vocab <= 4096
    assert _sampler(top_k=65) == _lib.Q3_ERR_UNSUPPORTED                          # k <= 64
    assert _sampler(vocab=32, row_stride=32, top_k=40) == _lib.Q3_ERR_INVALID     # k > vocab
    assert _sampler(temperature=0.0) == _lib.Q3_ERR_INVALID                       # sampling needs T > 0
    assert _sampler(logits_dtype=2) == _lib.Q3_ERR_INVALID
    assert _sampler(seen=512, seen_row_stride=3072) == _lib.Q3_ERR_INVALID        # seen rows need seat ids
    assert _sampler(emb=1024, emb_dim=1024, emb_row_stride=1024) == _lib.Q3_ERR_INVALID   # embedding without output
    assert _sampler(rng_state=132) == _lib.Q3_ERR_ALIGNMENT
    assert _sampler(batch=0) == _lib.Q3_OK


def test_row_kernels_reject_bad_arguments_before_cuda():
    lib = _lib.load()
    assert lib.q3_add_rms_norm(16, 1024, None, 0, 16, 16, 1024, 4, 1536, 1e-6, None) == _lib.Q3_ERR_UNSUPPORTED
    assert lib.q3_add_rms_norm(16, 512, None, 0, 16, 16, 1024, 4, 1024, 1e-6, None) == _lib.Q3_ERR_INVALID
    assert lib.q3_add_rms_norm(16, 1024, 24, 1024, 16, 16, 1024, 4, 1024, 1e-6, None) == _lib.Q3_ERR_ALIGNMENT
    assert lib.q3_add_rms_norm(None, 0, None, 0, None, None, 0, 0, 1024, 1e-6, None) == _lib.Q3_OK
    assert lib.q3_silu_mul(16, 6144, 16, 3072, 4, 3070, None) == _lib.Q3_ERR_INVALID     # ffn not a multiple of 8
    assert lib.q3_silu_mul(16, 4096, 16, 3072, 4, 3072, None) == _lib.Q3_ERR_INVALID     # row shorter than [g | u]
    assert lib.q3_silu_mul(24, 6144, 16, 3072, 4, 3072, None) == _lib.Q3_ERR_ALIGNMENT
    nr = _norm_rope()
    assert lib.q3_qk_norm_rope_rows(4096, 2048, ctypes.byref(nr), 4, None) == _lib.Q3_ERR_INVALID
    assert lib.q3_qk_norm_rope_rows(4096, 4096, None, 4, None) == _lib.Q3_ERR_INVALID
    assert lib.q3_qk_norm_rope_rows(4100, 4096, ctypes.byref(nr), 4, None) == _lib.Q3_ERR_ALIGNMENT


def test_prefix_copy_rejects_bad_arguments_before_cuda():
    lib = _lib.load()
    args = dict(k_src=16, v_src=16, ls=4096, ss=1024, kp=64, vp=64, L=28, rows=1024, page=16, nkv=8, hd=128,
                seat=128, slot=128, batch=2, plen=35, bt=256, bts=4, maxp=4)

    def call(**kw):
        a = dict(args)
        a.update(kw)
        return lib.q3_kv_copy_prefix(a["k_src"], a["v_src"], a["ls"], a["ss"], a["kp"], a["vp"], a["L"], a["rows"],
                                     a["page"], a["nkv"], a["hd"], a["seat"], a["slot"], a["batch"], a["plen"],
                                     a["bt"], a["bts"], a["maxp"], None)
    assert call(batch=-1) == _lib.Q3_ERR_INVALID
    assert call(seat=None) == _lib.Q3_ERR_INVALID
    assert call(bts=2) == _lib.Q3_ERR_INVALID                                     # table stride < pages per seat
    assert call(k_src=24) == _lib.Q3_ERR_ALIGNMENT
    assert call(L=0) == _lib.Q3_OK and call(plen=0) == _lib.Q3_OK


def test_prefill_rejects_bad_arguments_before_cuda():
    lib = _lib.load()
    base = dict(q=16, qs=2048, qr=640, k=16, v=16, kvs=1024, kvr=640, cuq=64, cuk=64, ns=2, mq=320, pl=None, seat=None,
                kp=32, vp=48, npg=100, page=16, bt=128, bts=20, maxp=20, wkv=0, causal=1, nh=16, nkv=8, hd=128, out=16,
                os_=2048)

    def call(**kw):
        a = dict(base)
        a.update(kw)
        return lib.q3_prefill(a["q"], a["qs"], a["qr"], a["k"], a["v"], a["kvs"], a["kvr"], a["cuq"], a["cuk"], a["ns"],
                              a["mq"], a["pl"],
                              a["seat"], a["kp"], a["vp"], a["npg"], a["page"], a["bt"], a["bts"], a["maxp"], a["wkv"],
                              a["causal"], a["nh"], a["nkv"], a["hd"], 0.088, a["out"], a["os_"], None)
    assert call(nh=32) == _lib.Q3_ERR_UNSUPPORTED                               # the model family: 16 / 8 x 128
    assert call(ns=-1) == _lib.Q3_ERR_INVALID
    assert call(cuq=None) == _lib.Q3_ERR_INVALID
    assert call(kvs=512) == _lib.Q3_ERR_INVALID                                 # K/V rows shorter than 8 x 128
    assert call(wkv=1, bt=None) == _lib.Q3_ERR_INVALID                          # page writes need a block table
    assert call(wkv=1, bts=10) == _lib.Q3_ERR_INVALID                           # table stride < pages per seat
    assert call(q=24) == _lib.Q3_ERR_ALIGNMENT
    assert call(ns=70000) == _lib.Q3_ERR_INVALID                                # beyond the grid's z extent
    assert call(qr=-1) == _lib.Q3_ERR_INVALID                                   # negative row counts
    assert call(kvr=-5) == _lib.Q3_ERR_INVALID
    assert call(qr=0) == _lib.Q3_OK                                             # no query rows: nothing to do
    assert call(ns=0) == _lib.Q3_OK


def test_cp_step_and_noalloc_reject_bad_arguments_before_cuda():
    lib = _lib.load()
    strides = (16384, 2048, 128, 16384, 2048, 128)
    assert lib.q3_cp_step(16, 2048, None, None, 1024, 16, 16, *strides, 4, 16, 2, 0.1, 16, 2048, None) == \
        _lib.Q3_ERR_INVALID                                                     # the new slot's k / v are required
    assert lib.q3_cp_step(16, 2048, 16, 16, 512, 16, 16, *strides, 4, 16, 2, 0.1, 16, 2048, None) == \
        _lib.Q3_ERR_INVALID                                                     # k / v rows shorter than 8 x 128
    assert lib.q3_cp_step(16, 2048, 20, 16, 1024, 16, 16, *strides, 4, 16, 2, 0.1, 16, 2048, None) == \
        _lib.Q3_ERR_ALIGNMENT
    assert lib.q3_paged_decode_noalloc(16, 2048, None, None, 0, 32, 32, 10, 16, 64, 64, 4, 4, -1, 16, 8, 128, 0.1,
                                       16, 2048, 0, None) == _lib.Q3_ERR_INVALID
    assert lib.q3_paged_decode_noalloc(16, 2048, None, None, 0, 32, 32, 10, 16, 64, 64, 4, 4, 2, 16, 8, 128, 0.1,
                                       16, 2048, -3, None) == _lib.Q3_ERR_INVALID


def test_noalloc_checks_every_argument_before_touching_cuda_or_its_scratch():
    """The allocation-free decode entry shares one scratch array between all calls on a device, so a call it refuses
    must queue nothing on it (no counter clearing that could hit a call in flight on another stream). Every argument
    check therefore runs before its first CUDA call: on a host without a GPU each bad call below returns its argument
    error, never Q3_ERR_CUDA, which is what any CUDA call would produce here."""
    lib = _lib.load()

    def call(q=16, kn=None, vn=None, kvs=0, kp=32, vp=32, pages=10, page=16, seq=64, bt=64, bts=4, mp=4, B=2,
             nh=16, nkv=8, hd=128, out=16, outs=2048, ns=0):
        return lib.q3_paged_decode_noalloc(q, 2048, kn, vn, kvs, kp, vp, pages, page, seq, bt, bts, mp, B, nh, nkv, hd,
                                           0.1, out, outs, ns, None)

    assert call(q=24) == _lib.Q3_ERR_ALIGNMENT                                  # q rows need 16-byte alignment
    assert call(kp=40) == _lib.Q3_ERR_ALIGNMENT
    assert call(nh=12) == _lib.Q3_ERR_UNSUPPORTED
    assert call(bt=None) == _lib.Q3_ERR_INVALID
    assert call(out=None) == _lib.Q3_ERR_INVALID
    assert call(outs=100) == _lib.Q3_ERR_INVALID                                # out rows shorter than 16 x 128
    assert call(kn=16) == _lib.Q3_ERR_INVALID                                   # k without v
    assert call(kn=16, vn=16, kvs=512) == _lib.Q3_ERR_ALIGNMENT                 # new rows shorter than 8 x 128
    assert call(B=0) == _lib.Q3_OK                                              # an empty batch does nothing at all


@pytest.mark.parametrize("name,valid,default", [("q3_set_ring_frame_kernel", range(0, 7), 6),
                                                ("q3_set_ring_chunk_kernel", range(0, 5), 1),
                                                ("q3_set_decode_variant", range(0, 6), 5),
                                                ("q3_set_prefill_kernel", range(0, 2), 0)])
def test_kernel_selectors_take_known_values_and_return_the_previous_one(name, valid, default):
    """The selectors are process-wide settings with no CUDA call: each returns the previous selection, takes every
    value it knows and leaves the selection unchanged for any other."""
    fn = getattr(_lib.load(), name)
    start = fn(default)                     # whatever an earlier test left, back to the default
    try:
        assert fn(default) == default
        for v in valid:
            fn(v)
            assert fn(v) == v
        last = valid[-1]
        for bad in (-1, valid[-1] + 1, 1000):
            assert fn(bad) == last          # refused: the selection stays
        assert fn(default) == last
    finally:
        fn(start)
