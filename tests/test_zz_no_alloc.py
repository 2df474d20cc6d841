"""GPU: the allocation-free decode entry point, q3_paged_decode_noalloc, called through the C ABI.

It is for callers that cannot allocate device memory for the split-K workspace -- hosts whose device memory belongs
to an arena they do not own, or call paths that must not allocate -- and uses a fixed 16 MiB scratch array compiled
into the library instead. Its results must match the workspace entry point q3_paged_decode on two calls in a row (the
second reusing the scratch the first left behind, with a larger batch and the fused append), and a batch beyond the
scratch must be refused before anything is launched.

This file is collected last so that a run stopping at its first failure has already run every other test; it also
passes alone in a fresh process.
"""
import ctypes

import pytest
import torch

from helpers import assert_close_attn, bits_equal
from q3attn import synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SCALE = 128 ** -0.5


@pytest.fixture(scope="module")
def q3():
    import q3attn
    q3attn._lib.load()
    return q3attn


def _noalloc(lib, q, kn, vn, kp, vp, seq, bt, out, num_splits=0):
    return lib.q3_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), None if kn is None else kn.data_ptr(), None if vn is None else vn.data_ptr(),
        0 if kn is None else kn.stride(0), kp.data_ptr(), vp.data_ptr(), kp.shape[0], kp.shape[1], seq.data_ptr(),
        bt.data_ptr(), bt.stride(0), bt.shape[1], q.shape[0], 16, 8, 128, ctypes.c_float(SCALE), out.data_ptr(),
        out.stride(0), num_splits, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("append_second", [True])
def test_noalloc_matches_workspace_entry_on_two_calls(q3, append_second):
    lib = q3._lib.load()
    q3._lib.read_status(clear=True)
    cases = [(81, 40, False, 0), (82, 300, append_second, 37)]   # (seed, seats, fused append, CTA count)
    for seed, B, append, splits in cases:
        lay = synth.paged_layout(seed, B=B, ctx_lo=1, ctx_hi=900, page=16, pages_per_seat=60)
        d = {k: v.to(DEV) for k, v in synth.decode_case(seed, lay, scale=0.5).items()}
        seq, bt = lay.ctx.to(DEV), lay.block_table.to(DEV)
        kp_ref, vp_ref = d["k_pool"].clone(), d["v_pool"].clone()
        if append:
            ref = q3.paged_decode_append(d["q"], d["k_new"], d["v_new"], kp_ref, vp_ref, seq, bt, SCALE, splits)
        else:
            ref = q3.paged_decode(d["q"], kp_ref, vp_ref, seq, bt, SCALE, splits)
        out = torch.full((B, 16, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
        rc = _noalloc(lib, d["q"], d["k_new"] if append else None, d["v_new"] if append else None,
                      d["k_pool"], d["v_pool"], seq, bt, out, splits)
        assert rc == q3._lib.Q3_OK, lib.q3_error_string(rc).decode()
        torch.cuda.synchronize()
        assert q3._lib.read_status(clear=True) == 0
        assert_close_attn(out, ref.float(), what=f"no-alloc call B={B} append={append}")
        if append:
            assert bits_equal(d["k_pool"], kp_ref) and bits_equal(d["v_pool"], vp_ref)


def test_noalloc_refuses_batch_beyond_scratch(q3):
    lib = q3._lib.load()
    B = 4096                                          # needs ~36 MB of workspace at the default grid
    lay = synth.paged_layout(83, B=8, ctx_lo=1, ctx_hi=16, page=16, pages_per_seat=1)
    d = {k: v.to(DEV) for k, v in synth.decode_case(83, lay).items()}
    q = torch.zeros((B, 16, 128), dtype=torch.bfloat16, device=DEV)
    seq = torch.ones(B, dtype=torch.int32, device=DEV)
    bt = torch.zeros((B, 1), dtype=torch.int32, device=DEV)
    out = torch.zeros((B, 16, 128), dtype=torch.bfloat16, device=DEV)
    rc = _noalloc(lib, q, None, None, d["k_pool"], d["v_pool"], seq, bt, out)
    assert rc == q3._lib.Q3_ERR_SCRATCH_LIMIT
    assert b"scratch" in lib.q3_error_string(rc)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0, "nothing may run when the call is refused"
