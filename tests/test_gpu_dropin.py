"""GPU: each of the reference engine's attention call sites, called through the q3attn drop-in exactly as the line
passes its arguments (same positional arguments, same keywords, same tensor views), at the reference's own layout:
256-token pages, the identity seat table seat_pages[s, j] = s * P + j, seat_len 768 (engine/talker.py:23-25, 42).

  engine/talker.py:72-77        index_copy_ appends + flash_attn_with_kvcache(q.unsqueeze(1), kc, vc, cache_seqlens=,
                                block_table=, softmax_scale=, causal=True), in a CUDA graph as the engine replays it
  engine/talker.py:152-169      packed prefill: index_copy_ of the prompt rows + flash_attn_varlen_func(q, k, v,
                                cu_seqlens_q=, cu_seqlens_k=, max_seqlen_q=, max_seqlen_k=, softmax_scale=, causal=True),
                                with v the strided view of the QKV rows that talker.py:160 passes
  engine/arrivals.py:141-148    flash_attn_func(q, K, V, softmax_scale=, causal=True) over the cat'ed prefix + new rows
  engine/code_predictor.py:58, 46-47   the slot write + the _post attention expression, replaced by
                                q3attn.cp_step(q, k, v, K[l, :B], V[l, :B], p, scale) on the [L, max_bs, 8, 16, 128]
                                scratch (code_predictor.py:20-21), and cp_attn(q, K, V, n_live, scale) (cp_attn.py:33)

Every output is held to the north-star bounds against the fp32 oracle; every K/V write is compared bit for bit with
the index_copy_ it replaces."""
import pytest
import torch

from helpers import assert_close_attn, bits_equal
from oracle import attention as OA
from q3attn import synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SCALE = 128 ** -0.5
SEAT_LEN, PAGE = 768, 256
P = SEAT_LEN // PAGE


@pytest.fixture(scope="module")
def q3():
    import q3attn
    q3attn._lib.load()
    return q3attn


def _engine_pools(n_seats, ctx, g):
    """kc / vc of one layer as Talker.__init__ allocates them ([(S+1)*P, 256, 8, 128], talker.py:30-31) with each
    seat's first ctx[s] positions filled, and the identity seat table (talker.py:42)."""
    S1 = n_seats + 1
    kc = torch.zeros(S1 * P, PAGE, 8, 128, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    pos = torch.arange(SEAT_LEN, device=DEV)
    fill = (pos[None, :] < ctx.to(DEV)[:, None]).view(S1 * P, PAGE, 1, 1)
    kc.copy_(synth.randn(kc.shape, g, 0.5, torch.bfloat16, DEV) * fill)
    vc.copy_(synth.randn(vc.shape, g, 0.5, torch.bfloat16, DEV) * fill)
    seat_pages = (torch.arange(S1, dtype=torch.int32, device=DEV)[:, None] * P
                  + torch.arange(P, dtype=torch.int32, device=DEV)[None, :]).contiguous()
    return kc, vc, seat_pages


def test_talker_decode_call_site(q3):
    """talker.py:107-112 + 72-77 for a bucket of 16 rows, 11 live seats, padded rows on the scratch seat."""
    from q3attn import flash_attn_with_kvcache
    n_seats, bucket, n_live = 12, 16, 11
    g = torch.Generator(device=DEV).manual_seed(5)
    gc = synth.cpu_gen(5)
    ctx = torch.zeros(n_seats + 1, dtype=torch.int64)
    live = torch.randperm(n_seats, generator=gc)[:n_live]
    ctx[live] = torch.tensor([1, 255, 256, 257, 511, 512, 600, 700, 766, 767, 300])[:n_live]
    kc, vc, seat_pages = _engine_pools(n_seats, ctx, g)
    pos_all = ctx.to(DEV)
    s_seat = torch.full((bucket,), n_seats, dtype=torch.int64, device=DEV)
    s_seat[:n_live] = live.to(DEV)
    q = synth.randn((bucket, 16, 128), g, 0.5, torch.bfloat16, DEV)
    k = synth.randn((bucket, 8, 128), g, 0.5, torch.bfloat16, DEV)
    v = synth.randn((bucket, 8, 128), g, 0.5, torch.bfloat16, DEV)
    for t in (q, k, v):          # padded rows all come from the scratch seat's one pending input: identical rows
        t[n_live + 1:] = t[n_live]
    kc0, vc0 = kc.clone(), vc.clone()

    def frame():
        seat = s_seat[:bucket]
        pos = pos_all[seat]
        slot, c, bt = seat * SEAT_LEN + pos, (pos + 1).to(torch.int32), seat_pages[seat]      # talker.py:108-110
        kc.view(-1, 8, 128).index_copy_(0, slot, k)                                            # talker.py:72
        vc.view(-1, 8, 128).index_copy_(0, slot, v)                                            # talker.py:73
        return flash_attn_with_kvcache(q.unsqueeze(1), kc, vc, cache_seqlens=c, block_table=bt, softmax_scale=SCALE,
                                       causal=True)                                           # talker.py:77

    out = frame()
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0
    assert out.shape == (bucket, 1, 16, 128)
    # the oracle: Talker._attn_ref's maths over the same pages (append first, then ctx + 1 keys)
    rk, rv = kc0.cpu(), vc0.cpu()
    seat = s_seat.cpu()
    ref = OA.decode_step(q.cpu(), k.cpu(), v.cpu(), rk, rv, ctx[seat].to(torch.int32), seat_pages.cpu()[seat], SCALE)
    assert_close_attn(out[:, 0], ref, what="talker.py:77")
    assert bits_equal(kc, rk) and bits_equal(vc, rv)
    # the same frame under CUDA-graph capture and replay, as the engine runs it (talker.py:115-137)
    st = torch.cuda.Stream(device=DEV)
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        frame()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            gout = frame()
    torch.cuda.current_stream().wait_stream(st)
    graph.replay()
    torch.cuda.synchronize()
    assert bits_equal(gout, out)
    # flash-attn's fused k/v append form (one launch instead of index_copy_ + attention) gives the same result
    kc.copy_(kc0)
    vc.copy_(vc0)
    seat = s_seat[:bucket]
    pos = pos_all[seat]
    fused = flash_attn_with_kvcache(q.unsqueeze(1), kc, vc, k=k.unsqueeze(1), v=v.unsqueeze(1),
                                    cache_seqlens=pos.to(torch.int32), block_table=seat_pages[seat],
                                    softmax_scale=SCALE, causal=True)
    torch.cuda.synchronize()
    assert bits_equal(kc, rk) and bits_equal(vc, rv)
    assert_close_attn(fused[:, 0], ref, what="talker.py:77 fused append")
    del graph


def test_talker_packed_prefill_call_site(q3):
    """Talker.prefill_hidden's attention (talker.py:149-169) for three prompts of one call: the rows written with
    index_copy_ at seat * seat_len + arange(L), then flash_attn_varlen_func with the exact keywords; k is the RoPE output
    (packed) and v the strided view of the QKV rows, as lines 158-160 pass them."""
    from q3attn import flash_attn_varlen_func
    seats, lens = [3, 0, 5], [37, 300, 5]
    n_seats = 6
    g = torch.Generator(device=DEV).manual_seed(6)
    kc, vc, _ = _engine_pools(n_seats, torch.zeros(n_seats + 1, dtype=torch.int64), g)
    T = sum(lens)
    qkv = synth.randn((T, 4096), g, 0.5, torch.bfloat16, DEV)           # [q 2048 | k 1024 | v 1024] per row
    q = qkv[:, :2048].reshape(T, 16, 128).clone()                         # rope() output: a fresh tensor
    k = qkv[:, 2048:3072].reshape(T, 8, 128).clone()
    v = qkv[:, 3072:].view(T, 8, 128)                                     # talker.py:160: a view, row stride 4096
    slot = torch.cat([s * SEAT_LEN + torch.arange(L, device=DEV) for s, L in zip(seats, lens)])   # talker.py:152
    cu = torch.tensor([0, 37, 337, 342], dtype=torch.int32, device=DEV)                             # talker.py:153
    kc.view(-1, 8, 128).index_copy_(0, slot, k)                                                   # talker.py:161
    vc.view(-1, 8, 128).index_copy_(0, slot, v)                                                   # talker.py:162
    o = flash_attn_varlen_func(q, k, v, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=max(lens),
                               max_seqlen_k=max(lens), softmax_scale=SCALE, causal=True)          # talker.py:169
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0
    ref = OA.prefill_varlen(q.cpu(), k.cpu(), v.contiguous().cpu(), cu.cpu(), SCALE)
    assert_close_attn(o, ref, what="talker.py:169")
    # the pages hold what the reference's index_copy_ put there, through the identity table
    for s, L, a in zip(seats, lens, cu.tolist()):
        got = kc.view(-1, 8, 128)[s * SEAT_LEN:s * SEAT_LEN + L]
        assert bits_equal(got, k[a:a + L])


def test_arrivals_prefix_prefill_call_site(q3):
    """FastAdmit._run's attention (arrivals.py:141-148): q [S, R] of the new positions over K = cat(prefix, new) with
    the exact call flash_attn_func(q, K, V, softmax_scale=T.scale, causal=True), causal aligned to the bottom right;
    then the flat-slot K/V write of all k + R positions (arrivals.py:144-145) through q3attn.kv_append_slots."""
    from q3attn import flash_attn_func, kv_append_slots
    S, k, R, n_seats = 4, 35, 42, 6
    g = torch.Generator(device=DEV).manual_seed(7)
    pk = synth.randn((S, k, 8, 128), g, 0.5, torch.bfloat16, DEV)
    pv = synth.randn((S, k, 8, 128), g, 0.5, torch.bfloat16, DEV)
    q = synth.randn((S, R, 16, 128), g, 0.5, torch.bfloat16, DEV)
    kk = synth.randn((S, R, 8, 128), g, 0.5, torch.bfloat16, DEV)
    qkv_v = synth.randn((S, R, 4096), g, 0.5, torch.bfloat16, DEV)
    vv = qkv_v[..., 3072:].view(S, R, 8, 128)                             # arrivals.py:118: a view of the QKV rows
    K, V = torch.cat((pk, kk), 1), torch.cat((pv, vv), 1)                 # arrivals.py:119
    o = flash_attn_func(q, K, V, softmax_scale=SCALE, causal=True)        # arrivals.py:148
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0
    ref = OA.prefill_prefix(q.cpu(), K.cpu(), V.cpu(), SCALE)
    assert_close_attn(o, ref, what="arrivals.py:148")
    kc, vc, _ = _engine_pools(n_seats, torch.zeros(n_seats + 1, dtype=torch.int64), g)
    seat = torch.tensor([4, 1, 0, 5], device=DEV)
    flat = (seat[:, None] * SEAT_LEN + torch.arange(k + R, device=DEV)[None, :]).reshape(-1)      # arrivals.py:139
    rk, rv = kc.clone(), vc.clone()
    rk.view(-1, 8, 128).index_copy_(0, flat, K.reshape(-1, 8, 128))                              # arrivals.py:144
    rv.view(-1, 8, 128).index_copy_(0, flat, V.reshape(-1, 8, 128))                              # arrivals.py:145
    kv_append_slots(K.reshape(-1, 8, 128), V.reshape(-1, 8, 128), kc, vc, flat)
    torch.cuda.synchronize()
    assert bits_equal(kc, rk) and bits_equal(vc, rv)


def test_code_predictor_call_site(q3):
    """CodePredictor._s (code_predictor.py:52-59) over the 16 slots of a frame, 5 layers, on the engine's scratch
    K/V [L, max_bs, 8, 16, 128] with a live batch B < max_bs (code_predictor.py:20-21, 56): the slot write of line 58
    and the attention of lines 46-47 become one q3attn.cp_step per (step, layer). k is the RoPE output and v the
    strided view of the QKV rows (code_predictor.py:41-42). The scratch must equal what index_copy_ writes, and the
    output must meet the bounds against the fp32 attention; cp_attn (cp_attn.py:33) on the written scratch too."""
    from q3attn import cp_attn, cp_step
    L, max_bs, B = 5, 16, 11
    g = torch.Generator(device=DEV).manual_seed(8)
    K = torch.zeros(L, max_bs, 8, 16, 128, dtype=torch.bfloat16, device=DEV)
    V = torch.zeros_like(K)
    RK, RV = K.clone(), V.clone()
    for p in range(16):
        pidx = torch.tensor([p], device=DEV)
        for l in range(L):
            qkv = synth.randn((B, 4096), g, 0.5, torch.bfloat16, DEV)
            q = qkv[:, :2048].reshape(B, 16, 128).clone()
            k = qkv[:, 2048:3072].reshape(B, 8, 128).clone()
            v = qkv[:, 3072:].view(B, 8, 128)
            o = cp_step(q, k, v, K[l, :B], V[l, :B], p, SCALE)
            RK[l, :B].index_copy_(2, pidx, k.unsqueeze(2))                 # code_predictor.py:58
            RV[l, :B].index_copy_(2, pidx, v.unsqueeze(2))
            torch.cuda.synchronize()
            assert bits_equal(K, RK) and bits_equal(V, RV), f"slot write p {p} layer {l}"
            ref = OA.cp_attention(q.cpu(), RK[l, :B].cpu(), RV[l, :B].cpu(), p + 1, SCALE)
            assert_close_attn(o, ref, what=f"code_predictor.py:46-47 p {p} l {l}")
            if l == 0:
                assert_close_attn(cp_attn(q, K[l, :B], V[l, :B], p + 1, SCALE), ref, what=f"cp_attn p {p}")
    assert q3._lib.read_status() == 0
    # the reference's own bf16 expression (code_predictor.py:46-47) on the final scratch, for scale: ours is closer to
    # the fp32 result than it
    mask = torch.full((16, 16), float("-inf"), device=DEV).triu(1).to(torch.bfloat16)
    q = synth.randn((B, 16, 128), g, 0.5, torch.bfloat16, DEV)
    att = torch.matmul(q.view(B, 8, 2, 128), K[0, :B].transpose(-1, -2)) * SCALE + mask[15]
    o_bf16 = torch.matmul(torch.softmax(att.float(), dim=-1).to(torch.bfloat16), V[0, :B]).reshape(B, 2048)
    ref = OA.cp_attention(q.cpu(), K[0, :B].cpu(), V[0, :B].cpu(), 16, SCALE)
    ours = cp_attn(q, K[0, :B], V[0, :B], 16, SCALE)
    e_ours = float((ours.float().cpu() - ref).abs().max())
    e_ref = float((o_bf16.float().cpu() - ref).abs().max())
    print(f"[dropin] cp max|d| vs fp32: q3attn {e_ours:.2e}, reference bf16 expression {e_ref:.2e}", flush=True)
    assert e_ours <= e_ref + 1e-3
