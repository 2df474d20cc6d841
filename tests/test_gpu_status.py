"""GPU: the failure reporting every pipeline kernel shares. A bounded wait that expires must raise
Q3_STATUS_WAIT_TIMEOUT and return, leaving the context usable for the next call. The wait is made to expire on
purpose, with an mbarrier that nothing arrives on; nothing faults, traps or waits without a limit."""
import ctypes

import pytest
import torch

from helpers import assert_close_attn
from oracle import attention as OA
from q3attn import synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def q3():
    import q3attn
    q3attn._lib.load()
    return q3attn


def test_expired_wait_reports_and_the_context_stays_usable(q3):
    lib = q3._lib.load()
    q3._lib.read_status(clear=True)
    torch.cuda.synchronize()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.q3_selftest_bounded_wait(ctypes.c_uint64(1_000_000), stream) == 0   # 1 ms
    torch.cuda.synchronize()
    assert q3._lib.read_status(clear=True) & q3._lib.STATUS_WAIT_TIMEOUT
    # limits outside 1 ns .. 100 ms are refused on the host, before any launch
    assert lib.q3_selftest_bounded_wait(ctypes.c_uint64(0), stream) != 0
    assert lib.q3_selftest_bounded_wait(ctypes.c_uint64(200_000_000), stream) != 0
    # the next call on the same context is correct and raises nothing
    lay = synth.paged_layout(3, B=6, ctx_lo=1, ctx_hi=300, page=16, pages_per_seat=20)
    d = synth.decode_case(3, lay, scale=0.5)
    dd = {k: v.to(DEV) for k, v in d.items()}
    out = q3.paged_decode(dd["q"], dd["k_pool"], dd["v_pool"], lay.ctx.to(DEV), lay.block_table.to(DEV), 128 ** -0.5, 0)
    torch.cuda.synchronize()
    assert q3._lib.read_status(clear=True) == 0
    ref = OA.decode_attention(d["q"], d["k_pool"], d["v_pool"], lay.ctx, lay.block_table, 128 ** -0.5)
    assert_close_attn(out, ref, what="decode after an expired wait")
