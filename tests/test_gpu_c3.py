"""GPU parity at BASELINE config 3's own shape: one 1.7B talker layer's attention, 470 decoding seats (ctx U[100,1500],
fused K/V append + paged decode, engine/talker.py:72-77) and 10 admitting seats chunk-prefilling 320-token prompts
into fresh pages (engine/talker.py:161-162 + 169 as one launch), on one stream and into the same per-layer pools --
the pair of launches `bench.py --workload c3` times. Checked against the fp32 oracle: 24 decode seats spread over the
batch, every prefill row, and every appended or prefilled K/V row bit for bit; then the same pair captured in a CUDA
graph and replayed must reproduce the eager outputs exactly."""
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


def test_c3_decode_and_chunked_prefill_into_shared_pools(q3):
    lay, pseats, plen = synth.c3_layout(3)
    nd, npf = 470, len(pseats)
    g = torch.Generator(device=DEV).manual_seed(3)
    shp = (lay.num_pages, 16, 8, 128)
    kp = synth.randn(shp, g, 0.5, torch.bfloat16, DEV)                # K, V ~ N(0,1) x 0.5
    vp = synth.randn(shp, g, 0.5, torch.bfloat16, DEV)
    qd = synth.randn((nd, 16, 128), g, 0.5, torch.bfloat16, DEV)
    kd = synth.randn((nd, 8, 128), g, 0.5, torch.bfloat16, DEV)
    vd = synth.randn((nd, 8, 128), g, 0.5, torch.bfloat16, DEV)
    T = npf * plen
    qp = synth.randn((T, 16, 128), g, 0.5, torch.bfloat16, DEV)
    kpn = synth.randn((T, 8, 128), g, 0.5, torch.bfloat16, DEV)
    vpn = synth.randn((T, 8, 128), g, 0.5, torch.bfloat16, DEV)
    bt = lay.block_table.to(DEV)
    btd = bt[:nd].contiguous()
    seq = lay.ctx[:nd].to(DEV)
    cu = torch.arange(npf + 1, dtype=torch.int32, device=DEV) * plen
    zeros = torch.zeros(npf, dtype=torch.int32, device=DEV)
    sid = torch.tensor(pseats, dtype=torch.int32, device=DEV)
    pick = torch.linspace(0, nd - 1, 24).long().tolist()
    # the pages the oracle reads, before the launches change them (the decode seats' K/V and the admitting seats')
    k0 = {b: kp[bt[b].long()].cpu() for b in pick}
    v0 = {b: vp[bt[b].long()].cpu() for b in pick}

    def layer():
        o_dec = q3.paged_decode_append(qd, kd, vd, kp, vp, seq, btd, SCALE, 0)
        o_pre = q3.prefill_paged(qp, kpn, vpn, kp, vp, cu, cu, plen, zeros, sid, bt, SCALE, True, True)
        return o_dec, o_pre

    poison_allocator((nd, 16, 128))
    poison_allocator((T, 16, 128))
    out_d, out_p = layer()
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0
    assert torch.isfinite(out_d.float()).all() and torch.isfinite(out_p.float()).all(), "an output row was never written"

    # every appended decode row sits at (seat, ctx) through the table, bit for bit
    rows = (bt[torch.arange(nd, device=DEV), (seq // 16).long()].long() * 16 + (seq % 16).long())
    assert bits_equal(kp.view(-1, 8, 128)[rows], kd) and bits_equal(vp.view(-1, 8, 128)[rows], vd), "decode appends"
    # every prefilled row of the 10 admitting seats, bit for bit
    for i, s in enumerate(pseats):
        pos = torch.arange(plen, device=DEV)
        r = bt[s, pos // 16].long() * 16 + pos % 16
        assert bits_equal(kp.view(-1, 8, 128)[r], kpn[i * plen:(i + 1) * plen]), f"prefill K rows of seat {s}"
        assert bits_equal(vp.view(-1, 8, 128)[r], vpn[i * plen:(i + 1) * plen]), f"prefill V rows of seat {s}"

    # decode outputs of 24 seats spread over the batch, against fp32 attention over the pages as they were + the append
    for b in pick:
        n = int(lay.ctx[b]) + 1
        kpool, vpool = k0[b].clone(), v0[b].clone()             # this seat's pages in table order
        tab = torch.arange(kpool.shape[0], dtype=torch.int32)[None]
        OA.append_paged(kpool, vpool, kd[b:b + 1].cpu(), vd[b:b + 1].cpu(), lay.ctx[b:b + 1], tab)
        ref = OA.decode_attention(qd[b:b + 1].cpu(), kpool, vpool, torch.tensor([n]), tab, SCALE)[0]
        assert_close_attn(out_d[b], ref, what=f"c3 decode seat {b} (ctx {n})")
    # prefill outputs: causal attention of each 320-token prompt over itself
    ref_p = OA.prefill_varlen(qp.cpu(), kpn.cpu(), vpn.cpu(), cu.cpu(), SCALE)
    assert_close_attn(out_p, ref_p, what="c3 chunked prefill")

    # the same pair of launches captured in a CUDA graph (as the bench replays it) reproduces the eager results
    s = torch.cuda.Stream(device=DEV)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer()                      # sizes this stream's decode workspace outside capture (rewrites the same rows)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            gd, gp = layer()
    torch.cuda.current_stream().wait_stream(s)
    graph.replay()
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0
    assert bits_equal(gd, out_d) and bits_equal(gp, out_p), "graph replay differs from the eager launches"
    del graph
