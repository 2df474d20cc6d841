"""GPU parity: tcgen05 prefill attention (engine/talker.py:169, engine/arrivals.py:148) and its fused page writes."""
import os

import numpy as np
import pytest
import torch

import make_golden as mg
from helpers import assert_close_attn, bits_equal, poison_allocator
from oracle import attention as OA
from q3attn import synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SCALE = 128 ** -0.5


@pytest.fixture(scope="module")
def q3():
    import q3attn
    q3attn._lib.load()
    return q3attn


@pytest.fixture(params=[0, 1], ids=["tma", "single"], autouse=True)
def prefill_kernel(q3, request):
    """Every test runs on both prefill kernels: the warp-specialised TMA kernel (default) and the single-warpgroup one
    (used for calls the TMA kernel does not fit)."""
    prev = q3.set_prefill_kernel(request.param)
    yield request.param
    q3.set_prefill_kernel(prev)


def _check_status(q3):
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0


@pytest.mark.parametrize("lens", [[1], [7, 63, 64, 65], [77], [130, 1, 200], [320] * 3])
def test_varlen_causal_matches_oracle(q3, lens):
    d = synth.prefill_case(sum(lens), lens)
    g = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}
    poison_allocator((sum(lens), 16, 128))
    out = q3.flash_attn_varlen_func(g["q"], g["k"], g["v"], g["cu_seqlens"], g["cu_seqlens"], max(lens), max(lens),
                                    softmax_scale=SCALE, causal=True)
    _check_status(q3)
    ref = OA.prefill_varlen(d["q"], d["k"], d["v"], d["cu_seqlens"], SCALE)
    assert_close_attn(out, ref, what=f"varlen {lens}")


def test_non_causal(q3):
    lens = [50, 129]
    d = synth.prefill_case(5, lens)
    g = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}
    out = q3.flash_attn_varlen_func(g["q"], g["k"], g["v"], g["cu_seqlens"], g["cu_seqlens"], max(lens), max(lens),
                                    softmax_scale=SCALE, causal=False)
    _check_status(q3)
    ref = torch.zeros(sum(lens), 16, 128)
    for i in range(len(lens)):
        a, b = int(d["cu_seqlens"][i]), int(d["cu_seqlens"][i + 1])
        qh = d["q"][a:b].float().permute(1, 0, 2).reshape(8, 2, b - a, 128)
        kh = d["k"][a:b].float().permute(1, 0, 2)[:, None]
        vh = d["v"][a:b].float().permute(1, 0, 2)[:, None]
        att = torch.softmax(torch.matmul(qh, kh.transpose(-1, -2)) * SCALE, -1)
        ref[a:b] = torch.matmul(att, vh).reshape(16, b - a, 128).permute(1, 0, 2)
    assert_close_attn(out, ref, what="non-causal")


@pytest.mark.parametrize("name", list(mg.PREFILL_CASES))
def test_flash_attn_func_bottom_right_against_reference(q3, golden_dir, name):
    """flash_attn_func(q [S,R], K [S,k+R]) with bottom-right causal alignment, against FastAdmit._attn_ref's output
    computed by the reference (engine/arrivals.py:125-131): at the north-star bounds on the bf16-rounded inputs the
    kernel sees, with the input rounding's share added to the max-abs bound on the original fp32 inputs."""
    g = np.load(os.path.join(golden_dir, "prefill.npz"))
    q, K, V = mg.prefill_inputs(*mg.PREFILL_CASES[name])
    out = q3.flash_attn_func(q.to(DEV, torch.bfloat16), K.to(DEV, torch.bfloat16), V.to(DEV, torch.bfloat16),
                             softmax_scale=SCALE, causal=True)
    _check_status(q3)
    assert_close_attn(out, torch.from_numpy(g[f"{name}_b16_out"]), what=f"golden {name} (bf16 inputs)")
    assert_close_attn(out, torch.from_numpy(g[f"{name}_out"]), atol=2e-2, what=f"golden {name} (fp32 inputs)")
    ref = OA.prefill_prefix(q.to(torch.bfloat16), K.to(torch.bfloat16), V.to(torch.bfloat16), SCALE)
    assert_close_attn(out, ref, what=f"oracle {name}")


@pytest.mark.parametrize("page", [8, 16, 32, 48, 256])
def test_paged_chunk_prefill_writes_pages_and_attends_over_prefix(q3, page):
    """Chunked prefill: sequence i has prefix_lens[i] tokens cached in its pages; its new rows are written at
    prefix_lens[i].. (bit-exact placement) and its queries attend over prefix + new (bottom-right causal)."""
    g = synth.cpu_gen(77 + page)
    seats, pps = 6, 512 // page
    bt = torch.randperm(seats * pps + 5, generator=g)[: seats * pps].view(seats, pps).to(torch.int32)
    kp = synth.randn((seats * pps + 5, page, 8, 128), g, 0.5, torch.bfloat16)
    vp = synth.randn((seats * pps + 5, page, 8, 128), g, 0.5, torch.bfloat16)
    seat_ids = torch.tensor([4, 0, 2, 5], dtype=torch.int32)
    prefix = torch.tensor([0, 35, 129, 300], dtype=torch.int32)
    lens = [70, 42, 64, 100]
    d = synth.prefill_case(9, lens, scale=0.5)
    T = sum(lens)
    gk, gv = kp.to(DEV), vp.to(DEV)
    out = q3.prefill_paged(d["q"].to(DEV), d["k"].to(DEV), d["v"].to(DEV), gk, gv, d["cu_seqlens"].to(DEV),
                           d["cu_seqlens"].to(DEV), max(lens), prefix.to(DEV), seat_ids.to(DEV), bt.to(DEV), SCALE, True,
                           True)
    _check_status(q3)
    rk, rv = kp.clone(), vp.clone()
    ref = torch.zeros(T, 16, 128)
    for i in range(len(lens)):
        a, b = int(d["cu_seqlens"][i]), int(d["cu_seqlens"][i + 1])
        s, P = int(seat_ids[i]), int(prefix[i])
        pos = torch.arange(P, P + (b - a), dtype=torch.int32)
        OA.append_paged(rk, rv, d["k"][a:b], d["v"][a:b], pos, bt[[s] * (b - a)])
        K = OA.gather_seat(rk, bt[s], P + b - a)
        V = OA.gather_seat(rv, bt[s], P + b - a)
        ref[a:b] = OA.prefill_prefix(d["q"][a:b][None], K[None], V[None], SCALE)[0]
    assert bits_equal(gk, rk) and bits_equal(gv, rv), "page writes not bit-exact"
    assert_close_attn(out, ref, what=f"paged prefill page {page}")


def test_c3_ten_prompts_of_320_tokens_into_fresh_pages(q3):
    """BASELINE config 3's admission part: 10 seats each prefilling a 320-token prompt into fresh pages (page 16)."""
    lay, seats, L = synth.c3_layout(3)
    n = len(seats)
    d = synth.prefill_case(33, [L] * n, scale=0.5)
    pps = lay.block_table.shape[1]
    kp = torch.zeros(lay.num_pages, 16, 8, 128, dtype=torch.bfloat16, device=DEV)
    vp = torch.zeros_like(kp)
    out = q3.prefill_paged(d["q"].to(DEV), d["k"].to(DEV), d["v"].to(DEV), kp, vp, d["cu_seqlens"].to(DEV),
                           d["cu_seqlens"].to(DEV), L, torch.zeros(n, dtype=torch.int32, device=DEV),
                           torch.tensor(seats, dtype=torch.int32, device=DEV), lay.block_table.to(DEV), SCALE, True, True)
    _check_status(q3)
    ref = OA.prefill_varlen(d["q"], d["k"], d["v"], d["cu_seqlens"], SCALE)
    assert_close_attn(out, ref, what="c3 prefill")
    for i, s in enumerate(seats[:3]):
        got = OA.gather_seat(kp.cpu(), lay.block_table[s], L).to(torch.bfloat16)
        assert bits_equal(got, d["k"][i * L:(i + 1) * L]), f"seat {s} pages"
    assert pps * 16 >= L


@pytest.mark.parametrize("page", [16, 256])
def test_stale_non_finite_rows_never_reach_the_output(q3, page):
    """Page rows past each sequence's prefix and packed K/V rows that belong to no sequence hold NaN / inf: the
    attention reads whole tiles, but such rows get zero weight and must not leak (0 * NaN) into any output."""
    g = synth.cpu_gen(5 + page)
    seats, pps = 3, 512 // page
    n_pages = seats * pps
    bt = torch.randperm(n_pages, generator=g).view(seats, pps).to(torch.int32)
    kp = synth.randn((n_pages, page, 8, 128), g, 0.5, torch.bfloat16)
    vp = synth.randn((n_pages, page, 8, 128), g, 0.5, torch.bfloat16)
    prefix = torch.tensor([35, 100, 1], dtype=torch.int32)
    seat_ids = torch.tensor([2, 0, 1], dtype=torch.int32)
    for s_, P in zip(seat_ids.tolist(), prefix.tolist()):    # everything past the prefix in the seat's pages: NaN / inf
        pos = torch.arange(P, pps * page)
        rows = bt[s_, pos // page].long() * page + pos % page
        kp.view(-1, 8, 128)[rows] = float("nan")
        vp.view(-1, 8, 128)[rows] = float("inf")
    lens = [42, 20, 70]
    d = synth.prefill_case(13, lens, scale=0.5)
    pad = 40                                                  # packed rows after the last sequence: NaN
    k = torch.cat([d["k"], torch.full((pad, 8, 128), float("nan"), dtype=torch.bfloat16)])
    v = torch.cat([d["v"], torch.full((pad, 8, 128), float("nan"), dtype=torch.bfloat16)])
    out = q3.prefill_paged(d["q"].to(DEV), k.to(DEV), v.to(DEV), kp.to(DEV), vp.to(DEV), d["cu_seqlens"].to(DEV),
                           d["cu_seqlens"].to(DEV), max(lens), prefix.to(DEV), seat_ids.to(DEV), bt.to(DEV), SCALE, True,
                           False)
    _check_status(q3)
    assert torch.isfinite(out.float()).all()
    ref = torch.zeros(sum(lens), 16, 128)
    for i in range(len(lens)):
        a, b = int(d["cu_seqlens"][i]), int(d["cu_seqlens"][i + 1])
        P = int(prefix[i])
        K = torch.cat([OA.gather_seat(kp, bt[int(seat_ids[i])], P), d["k"][a:b].float()])
        V = torch.cat([OA.gather_seat(vp, bt[int(seat_ids[i])], P), d["v"][a:b].float()])
        ref[a:b] = OA.prefill_prefix(d["q"][a:b][None], K[None], V[None], SCALE)[0]
    assert_close_attn(out, ref, what=f"stale rows, page {page}")
