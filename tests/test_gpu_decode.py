"""GPU parity: paged decode attention and the K/V appends against the CPU oracle (restating engine/talker.py:72-88)."""
import os

import numpy as np
import pytest
import torch

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


def _to(d, dev=DEV):
    return {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in d.items()}


def _layout(B, ctx, page, pps, num_pages=None, seed=0):
    g = synth.cpu_gen(seed)
    num_pages = num_pages or B * pps
    perm = torch.randperm(num_pages, generator=g)[: B * pps]
    return synth.PagedLayout(ctx=torch.as_tensor(ctx, dtype=torch.int32), block_table=perm.view(B, pps).to(torch.int32),
                             page=page, num_pages=num_pages)


def _run_decode(q3, lay, d, append, num_splits=0):
    dd = _to(d)
    seq = lay.ctx.to(DEV)
    bt = lay.block_table.to(DEV)
    poison_allocator((lay.B, 16, 128))
    if append:
        out = q3.paged_decode_append(dd["q"], dd["k_new"], dd["v_new"], dd["k_pool"], dd["v_pool"], seq, bt, SCALE, num_splits)
    else:
        out = q3.paged_decode(dd["q"], dd["k_pool"], dd["v_pool"], seq, bt, SCALE, num_splits)
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0
    return out, dd


def _oracle(lay, d, append):
    kp, vp = d["k_pool"].clone(), d["v_pool"].clone()
    if append:
        o = OA.decode_step(d["q"], d["k_new"], d["v_new"], kp, vp, lay.ctx, lay.block_table, SCALE)
    else:
        o = OA.decode_attention(d["q"], kp, vp, lay.ctx, lay.block_table, SCALE)
    return o, kp, vp


@pytest.mark.parametrize("seed", [1, 11, 12])
@pytest.mark.parametrize("append", [False, True])
def test_decode_c1(q3, seed, append):
    """BASELINE config 1 layout (4 seats, ctx U[1,256], page 16, 128-page shuffled pool), bf16 inputs."""
    lay = synth.c1_layout(seed)
    if append:
        lay.ctx = lay.ctx - 1                       # the appended token brings the attended length back to ctx
    d = synth.decode_case(seed, lay, scale=1.0)
    out, dd = _run_decode(q3, lay, d, append)
    ref, kp, vp = _oracle(lay, d, append)
    assert_close_attn(out, ref, what=f"c1 seed {seed} append {append}")
    if append:
        assert bits_equal(dd["k_pool"], kp) and bits_equal(dd["v_pool"], vp), "append placement not bit-exact"


def test_decode_c1_against_reference_golden(q3, golden_dir):
    """The GPU kernel against the reference's own Talker._attn_ref output: at the north-star bounds against the
    reference run on the bf16-rounded inputs the kernel sees, and against the reference on the original fp32 inputs
    with the input rounding's share added to the max-abs bound (rounding N(0,1) inputs to bf16 moves outputs by up to
    ~1e-2 by itself)."""
    import make_golden as mg
    g = np.load(os.path.join(golden_dir, "decode_c1.npz"))
    for seed in (1, 11, 12):
        lay, d = mg.c1_inputs(seed)
        out, _ = _run_decode(q3, lay, {k: v.to(torch.bfloat16) for k, v in d.items()}, append=False)
        assert_close_attn(out, torch.from_numpy(g[f"s{seed}_b16_out"]), what=f"golden seed {seed} (bf16 inputs)")
        assert_close_attn(out, torch.from_numpy(g[f"s{seed}_out"]), atol=2e-2, what=f"golden seed {seed} (fp32 inputs)")


EDGE_CTX = [1, 2, 15, 16, 17, 31, 32, 33, 255, 256, 257]


@pytest.mark.parametrize("page", [1, 8, 16, 32, 256])
@pytest.mark.parametrize("append", [False, True])
def test_decode_edge_lengths(q3, page, append):
    pps = (512 + page - 1) // page
    ctx = [c - 1 if append else c for c in EDGE_CTX] + ([pps * page - 1] if append else [pps * page])
    lay = _layout(len(ctx), ctx, page, pps, num_pages=len(ctx) * pps + 7, seed=page)
    d = synth.decode_case(100 + page, lay, scale=0.5)
    out, dd = _run_decode(q3, lay, d, append)
    ref, kp, vp = _oracle(lay, d, append)
    assert_close_attn(out, ref, what=f"page {page} append {append}")
    if append:
        assert bits_equal(dd["k_pool"], kp) and bits_equal(dd["v_pool"], vp)


@pytest.mark.parametrize("num_splits", [1, 2, 3, 7, 148, 1000])
def test_decode_split_counts(q3, num_splits):
    """Any CTA count gives the same answer (seats straddling 1..many CTAs, merged by the last arrival)."""
    lay = synth.paged_layout(5, B=9, ctx_lo=1, ctx_hi=700, page=16, pages_per_seat=44)
    d = synth.decode_case(5, lay, scale=0.5)
    out, _ = _run_decode(q3, lay, d, append=True, num_splits=num_splits)
    lay.ctx = lay.ctx.clone()
    ref, _, _ = _oracle(lay, d, append=True)
    assert_close_attn(out, ref, what=f"splits {num_splits}")


@pytest.mark.parametrize("variant", [0, 2, 3, 4, 5])
def test_decode_pair_weighted_split(q3, variant):
    """The default grid of the two-CTAs-per-SM variants (pair-weighted chunk split: the first CTA resident on each SM
    takes a larger share) with enough chunks to engage it; every seat checked, seats straddling CTAs of both weights.
    Variant 5 (two chunk streams per CTA, uniform split) runs its own default grid through the same check."""
    prev = q3.set_decode_variant(variant)
    try:
        lay = synth.paged_layout(21, B=128, ctx_lo=100, ctx_hi=700, page=16, pages_per_seat=44)
        d = synth.decode_case(21, lay, scale=0.5)
        out, dd = _run_decode(q3, lay, d, append=True)
        ref, kp, vp = _oracle(lay, d, append=True)
        assert_close_attn(out, ref, what=f"pair split variant {variant}")
        assert bits_equal(dd["k_pool"], kp) and bits_equal(dd["v_pool"], vp)
    finally:
        q3.set_decode_variant(prev)


def test_decode_empty_seats_give_zero(q3):
    lay = _layout(4, [0, 5, 0, 40], 16, 4, seed=3)
    d = synth.decode_case(3, lay)
    out, _ = _run_decode(q3, lay, d, append=False)
    assert torch.count_nonzero(out[0].float()) == 0 and torch.count_nonzero(out[2].float()) == 0
    ref, _, _ = _oracle(lay, d, append=False)
    assert_close_attn(out, ref, what="empty seats")


def test_decode_c2_full_size_subset(q3):
    """BASELINE config 2 at full size (576 seats, ctx U[200,1200], 43,776-page shuffled pool), one layer with the fused
    append; the oracle checks 24 seats spread over the batch and every appended row."""
    lay = synth.c2_layout(2)
    B = lay.B
    g = torch.Generator(device=DEV).manual_seed(2)
    shp = (lay.num_pages, lay.page, 8, 128)
    kp = synth.randn(shp, g, 0.5, torch.bfloat16, DEV)
    vp = synth.randn(shp, g, 0.5, torch.bfloat16, DEV)
    q = synth.randn((B, 16, 128), g, 0.5, torch.bfloat16, DEV)
    kn = synth.randn((B, 8, 128), g, 0.5, torch.bfloat16, DEV)
    vn = synth.randn((B, 8, 128), g, 0.5, torch.bfloat16, DEV)
    seq, bt = lay.ctx.to(DEV), lay.block_table.to(DEV)
    poison_allocator((B, 16, 128))
    out = q3.paged_decode_append(q, kn, vn, kp, vp, seq, bt, SCALE, 0)
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0
    assert torch.isfinite(out.float()).all(), "some seat's output was never written"
    pick = torch.linspace(0, B - 1, 24).long()
    for b in pick.tolist():
        n = int(lay.ctx[b]) + 1
        rows = bt[b, : (n + 15) // 16].long()
        K = kp[rows].reshape(-1, 8, 128)[:n].float().cpu()
        V = vp[rows].reshape(-1, 8, 128)[:n].float().cpu()
        assert bits_equal(K[n - 1].to(torch.bfloat16), kn[b].cpu()) and bits_equal(V[n - 1].to(torch.bfloat16), vn[b].cpu())
        a = torch.matmul(q[b].float().cpu().view(8, 2, 128), K.transpose(0, 1).transpose(-1, -2)) * SCALE
        ref = torch.matmul(torch.softmax(a, -1), V.transpose(0, 1)).reshape(16, 128)
        assert_close_attn(out[b], ref, what=f"c2 seat {b}")


@pytest.mark.parametrize("variant", [0, 1, 2, 3, 4, 5])
def test_decode_every_kernel_variant(q3, variant):
    """Every decode kernel variant (8/16-token chunks, 2/3 stages) against the oracle on edge lengths with 16-token
    pages, a 1-token page layout and 256-token pages, with and without the fused append."""
    prev = q3.set_decode_variant(variant)
    try:
        for page, append in ((16, True), (16, False), (1, True), (256, False)):
            pps = (512 + page - 1) // page
            ctx = [c - 1 if append else c for c in EDGE_CTX] + ([pps * page - 1] if append else [pps * page])
            lay = _layout(len(ctx), ctx, page, pps, num_pages=len(ctx) * pps + 3, seed=7 + page)
            d = synth.decode_case(200 + page, lay, scale=0.5)
            out, dd = _run_decode(q3, lay, d, append, num_splits=37)
            ref, kp, vp = _oracle(lay, d, append)
            assert_close_attn(out, ref, what=f"variant {variant} page {page} append {append}")
            if append:
                assert bits_equal(dd["k_pool"], kp) and bits_equal(dd["v_pool"], vp)
    finally:
        q3.set_decode_variant(prev)


@pytest.mark.parametrize("num_splits", [1, 2, 3, 295, 296, 1000])
def test_decode_producer_streams_split_counts(q3, num_splits):
    """The dedicated-producer variant (two chunk streams per CTA) at any stream count, odd ones included (the last
    CTA's second stream then has no chunk), with the fused append."""
    prev = q3.set_decode_variant(5)
    try:
        lay = synth.paged_layout(15, B=40, ctx_lo=1, ctx_hi=900, page=16, pages_per_seat=60)
        d = synth.decode_case(15, lay, scale=0.5)
        out, dd = _run_decode(q3, lay, d, append=True, num_splits=num_splits)
        ref, kp, vp = _oracle(lay, d, append=True)
        assert_close_attn(out, ref, what=f"producer streams, splits {num_splits}")
        assert bits_equal(dd["k_pool"], kp) and bits_equal(dd["v_pool"], vp)
        assert q3._lib.read_status() == 0
    finally:
        q3.set_decode_variant(prev)


def test_workspace_reuse_across_batches_and_splits(q3):
    """One workspace serves launches of any batch and split count in any order: a launch that leaves partials behind
    (many splits, small batch) must not disturb the ticket counters of a later, larger launch."""
    seqs = [(3, 1000), (40, 0), (5, 300), (64, 0), (2, 7), (64, 148)]
    for i, (B, splits) in enumerate(seqs):
        lay = synth.paged_layout(60 + i, B=B, ctx_lo=1, ctx_hi=600, page=16, pages_per_seat=40)
        d = synth.decode_case(60 + i, lay, scale=0.5)
        out, _ = _run_decode(q3, lay, d, append=False, num_splits=splits)
        ref, _, _ = _oracle(lay, d, append=False)
        assert_close_attn(out, ref, what=f"launch {i} (B {B}, splits {splits})")


def test_kv_append_slots_bit_exact(q3):
    g = synth.cpu_gen(9)
    pool_k = synth.randn((64, 16, 8, 128), g, 1.0, torch.bfloat16)
    pool_v = synth.randn((64, 16, 8, 128), g, 1.0, torch.bfloat16)
    k = synth.randn((100, 8, 128), g, 1.0, torch.bfloat16)
    v = synth.randn((100, 8, 128), g, 1.0, torch.bfloat16)
    slots = torch.randperm(64 * 16, generator=g)[:100]
    rk, rv = pool_k.clone(), pool_v.clone()
    OA.append_slots(rk, rv, k, v, slots)
    gk, gv = pool_k.to(DEV), pool_v.to(DEV)
    q3.kv_append_slots(k.to(DEV), v.to(DEV), gk, gv, slots.to(DEV))
    torch.cuda.synchronize()
    assert bits_equal(gk, rk) and bits_equal(gv, rv)


def test_kv_append_paged_bit_exact_and_identity_table_flat(q3):
    """Paged placement through a shuffled table, and through the reference's identity table with 256-token pages it
    lands exactly at seat*seat_len + pos (engine/talker.py:42, 72-73, 109)."""
    g = synth.cpu_gen(10)
    S1, seat_len = 9, 512
    P = seat_len // 256
    for page, bt in ((16, torch.randperm(S1 * 32, generator=g).view(S1, 32).to(torch.int32)),
                     (256, (torch.arange(S1)[:, None] * P + torch.arange(P)[None, :]).to(torch.int32))):
        npg = int(bt.numel())
        pk = synth.randn((npg, page, 8, 128), g, 1.0, torch.bfloat16)
        pv = synth.randn((npg, page, 8, 128), g, 1.0, torch.bfloat16)
        k = synth.randn((S1, 8, 128), g, 1.0, torch.bfloat16)
        v = synth.randn((S1, 8, 128), g, 1.0, torch.bfloat16)
        pos = torch.randint(0, seat_len, (S1,), generator=g).to(torch.int32)
        rk, rv = pk.clone(), pv.clone()
        OA.append_paged(rk, rv, k, v, pos, bt)
        if page == 256:
            fk = pk.clone()
            fk.view(-1, 8, 128).index_copy_(0, torch.arange(S1) * seat_len + pos.long(), k)
            assert bits_equal(fk, rk)
        gk, gv = pk.to(DEV), pv.to(DEV)
        q3.kv_append_paged(k.to(DEV), v.to(DEV), gk, gv, pos.to(DEV), bt.to(DEV))
        torch.cuda.synchronize()
        assert bits_equal(gk, rk) and bits_equal(gv, rv)


def test_bad_block_table_entry_reports_status(q3):
    """An out-of-range page id is caught by the kernel's own bounds check (clamped, status bit raised)."""
    lay = _layout(2, [20, 20], 16, 2, seed=4)
    lay.block_table[1, 1] = 10_000
    d = synth.decode_case(4, lay)
    dd = _to(d)
    q3._lib.read_status(clear=True)
    q3.paged_decode(dd["q"], dd["k_pool"], dd["v_pool"], lay.ctx.to(DEV), lay.block_table.to(DEV), SCALE, 0)
    torch.cuda.synchronize()
    assert q3._lib.read_status(clear=True) & q3._lib.STATUS_BAD_PAGE


def test_flash_api_dropin_matches_oracle(q3):
    """flash_attn_with_kvcache signature as used at engine/talker.py:77 (q [B,1,16,128], paged caches)."""
    lay = synth.c1_layout(1)
    d = synth.decode_case(1, lay)
    dd = _to(d)
    poison_allocator((4, 16, 128))
    out = q3.flash_attn_with_kvcache(dd["q"].unsqueeze(1), dd["k_pool"], dd["v_pool"], cache_seqlens=lay.ctx.to(DEV),
                                     block_table=lay.block_table.to(DEV), softmax_scale=SCALE, causal=True)
    ref, _, _ = _oracle(lay, d, append=False)
    assert out.shape == (4, 1, 16, 128)
    assert_close_attn(out[:, 0], ref, what="flash api")
    # non-paged cache [B, S, 8, 128] + fused k/v append
    B, S = 3, 300
    g = synth.cpu_gen(2)
    kc = synth.randn((B, S, 8, 128), g, 0.5, torch.bfloat16)
    vc = synth.randn((B, S, 8, 128), g, 0.5, torch.bfloat16)
    q = synth.randn((B, 1, 16, 128), g, 0.5, torch.bfloat16)
    k = synth.randn((B, 1, 8, 128), g, 0.5, torch.bfloat16)
    v = synth.randn((B, 1, 8, 128), g, 0.5, torch.bfloat16)
    seq = torch.tensor([0, 150, 299], dtype=torch.int32)
    gk, gv = kc.to(DEV), vc.to(DEV)
    out = q3.flash_attn_with_kvcache(q.to(DEV), gk, gv, k=k.to(DEV), v=v.to(DEV), cache_seqlens=seq.to(DEV),
                                     softmax_scale=SCALE, causal=True)
    rk, rv = kc.clone().view(B, 1, S, 8, 128).flatten(0, 1), vc.clone().view(B, 1, S, 8, 128).flatten(0, 1)
    ref = OA.decode_step(q[:, 0], k[:, 0], v[:, 0], rk, rv, seq, torch.arange(B, dtype=torch.int32)[:, None], SCALE)
    assert_close_attn(out[:, 0], ref, what="flash api contiguous cache")
    assert bits_equal(gk, rk.view(B, S, 8, 128)) and bits_equal(gv, rv.view(B, S, 8, 128))


def test_cuda_graph_replay_matches_eager(q3):
    """The op records into a CUDA graph (no host sync, no allocation after warm-up) and replays with new inputs."""
    lay = synth.paged_layout(6, B=16, ctx_lo=1, ctx_hi=300, page=16, pages_per_seat=20)
    d = _to(synth.decode_case(6, lay))
    seq, bt = lay.ctx.to(DEV), lay.block_table.to(DEV)
    kp0, vp0 = d["k_pool"].clone(), d["v_pool"].clone()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(2):
            q3.paged_decode(d["q"], d["k_pool"], d["v_pool"], seq, bt, SCALE, 0)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = q3.paged_decode_append(d["q"], d["k_new"], d["v_new"], d["k_pool"], d["v_pool"], seq, bt, SCALE, 0)
    for step in range(3):
        d["q"].copy_(synth.randn(d["q"].shape, synth.cpu_gen(50 + step), 0.5, torch.bfloat16))
        d["k_pool"].copy_(kp0)
        d["v_pool"].copy_(vp0)
        g.replay()
        torch.cuda.synchronize()
        kp, vp = kp0.clone(), vp0.clone()
        ref = q3.paged_decode_append(d["q"], d["k_new"], d["v_new"], kp, vp, seq, bt, SCALE, 0)
        torch.cuda.synchronize()
        assert bits_equal(out, ref) and bits_equal(kp, d["k_pool"])
    del g
