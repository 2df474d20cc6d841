"""GPU parity: q/k RMSNorm + RoPE fused into the attention kernels (engine/ops.py:51-60 as called at
engine/talker.py:69-71 and engine/code_predictor.py:40-42).

Two comparators per case:
  * the reference's own eager ops in bf16 (oracle.frame.rms / rope, the restatement of ops.py:51-60) feeding the
    already-verified unfused kernels: the fused kernels must produce the same appended rows (v bit-exact; k equal
    except for rare one-ulp flips where the fp32 sum of squares is rounded in a different order) and the same outputs;
  * the fp32 oracle attention over those q/k/v, within the attention tolerance."""
import pytest
import torch

from helpers import assert_close_attn, bits_equal, poison_allocator
from oracle import attention as OA
from oracle import frame as OF
from q3attn import synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SCALE = 128 ** -0.5
NQ, NK = 16 * 128, 8 * 128


@pytest.fixture(scope="module")
def q3():
    import q3attn
    q3attn._lib.load()
    return q3attn


def rope_tables(n_pos: int, base: float = 1e6):
    """Rotate-half rotary tables [n_pos, 128] (bf16), as rotary_emb builds them (cat(freqs, freqs))."""
    inv = 1.0 / (base ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    f = torch.arange(n_pos, dtype=torch.float32)[:, None] * inv[None, :]
    e = torch.cat([f, f], -1)
    return e.cos().to(torch.bfloat16), e.sin().to(torch.bfloat16)


def norm_weights(seed: int):
    g = synth.cpu_gen(seed)
    qn = (1.0 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    kn = (1.0 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    return qn, kn


def eager_split(qkv, qn, kn, cos, sin):
    """q, k, v (contiguous) of one layer with the reference's eager bf16 ops (talker.py:69-71); cos/sin [B,128] or
    [128]."""
    B = qkv.shape[0]
    c = cos.view(-1, 1, 128)
    s = sin.view(-1, 1, 128)
    q = OF.rope(OF.rms(qkv[:, :NQ].view(B, 16, 128), qn), c, s)
    k = OF.rope(OF.rms(qkv[:, NQ:NQ + NK].view(B, 8, 128), kn), c, s)
    v = qkv[:, NQ + NK:].reshape(B, 8, 128).contiguous()
    return q.contiguous(), k.contiguous(), v


def ulp_flips(a: torch.Tensor, b: torch.Tensor):
    """(count of differing bf16 values, largest difference in units of the last place) between two bf16 tensors."""
    ai = a.contiguous().view(torch.int16).to(torch.int32)
    bi = b.contiguous().view(torch.int16).to(torch.int32)
    d = (ai - bi).abs()
    return int((d != 0).sum()), int(d.max()) if d.numel() else 0


@pytest.mark.parametrize("page,shared_rope", [(16, False), (1, False), (256, False), (16, True)])
def test_fused_decode_layer_matches_eager_ops(q3, page, shared_rope):
    pps = (512 + page - 1) // page
    ctx = [0, 1, 15, 16, 31, 255, 256, 300, 510, pps * page - 1]
    B = len(ctx)
    g = synth.cpu_gen(40 + page)
    perm = torch.randperm(B * pps + 5, generator=g)[: B * pps]
    bt = perm.view(B, pps).to(torch.int32)
    seq = torch.tensor(ctx, dtype=torch.int32)
    kp = synth.randn((B * pps + 5, page, 8, 128), g, 0.5, torch.bfloat16)
    vp = synth.randn((B * pps + 5, page, 8, 128), g, 0.5, torch.bfloat16)
    qkv = synth.randn((B, NQ + 2 * NK), g, 1.0, torch.bfloat16)
    qn, kn = norm_weights(41 + page)
    ct, st = rope_tables(pps * page)
    cos, sin = (ct[300], st[300]) if shared_rope else (ct[seq.long()], st[seq.long()])

    d = {k: t.to(DEV) for k, t in dict(qkv=qkv, qn=qn, kn=kn, cos=cos, sin=sin, seq=seq, bt=bt).items()}
    kp_a, vp_a, kp_b, vp_b = kp.to(DEV), vp.to(DEV), kp.to(DEV), vp.to(DEV)
    q, k, v = eager_split(d["qkv"], d["qn"], d["kn"], d["cos"], d["sin"])
    out_a = q3.paged_decode_append(q, k, v, kp_a, vp_a, d["seq"], d["bt"], SCALE)
    poison_allocator((B, 16, 128))
    out_b = q3.paged_decode_qkv(d["qkv"], d["qn"], d["kn"], d["cos"], d["sin"], kp_b, vp_b, d["seq"], d["bt"], SCALE)
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0

    assert bits_equal(vp_b, vp_a), "v rows (raw projection) must be appended bit-exactly"
    n, worst = ulp_flips(kp_b, kp_a)
    assert worst <= 1 and n <= max(2, B * 1024 // 200), f"appended k rows: {n} values differ, up to {worst} ulp"
    assert_close_attn(out_b, out_a, what=f"fused vs eager-composed page {page}")
    ref = OA.decode_step(q.cpu(), k.cpu(), v.cpu(), kp.clone(), vp.clone(), seq, bt, SCALE)
    assert_close_attn(out_b, ref, what=f"fused vs fp32 oracle page {page}")


def test_fused_decode_c2_shape(q3):
    """BASELINE config 2 shapes (576 seats, ctx U[200,1200], page 16, shuffled table): fused layer vs eager ops."""
    lay = synth.c2_layout(2)
    g = synth.cpu_gen(52)
    qkv = synth.randn((lay.B, NQ + 2 * NK), g, 1.0, torch.bfloat16).to(DEV)
    qn, kn = (t.to(DEV) for t in norm_weights(53))
    ct, st = rope_tables(1216)
    seq = lay.ctx.to(DEV)
    cos, sin = ct.to(DEV)[seq.long()], st.to(DEV)[seq.long()]
    gd = torch.Generator(device=DEV).manual_seed(54)
    kp = torch.randn((lay.num_pages, 16, 8, 128), generator=gd, device=DEV).mul_(0.5).to(torch.bfloat16)
    vp = torch.randn((lay.num_pages, 16, 8, 128), generator=gd, device=DEV).mul_(0.5).to(torch.bfloat16)
    bt = lay.block_table.to(DEV)
    kp_b, vp_b = kp.clone(), vp.clone()
    q, k, v = eager_split(qkv, qn, kn, cos, sin)
    out_a = q3.paged_decode_append(q, k, v, kp, vp, seq, bt, SCALE)
    out_b = q3.paged_decode_qkv(qkv, qn, kn, cos, sin, kp_b, vp_b, seq, bt, SCALE)
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0
    assert bits_equal(vp_b, vp)
    n, worst = ulp_flips(kp_b, kp)
    assert worst <= 1 and n <= lay.B * 1024 // 200, f"appended k rows: {n} values differ, up to {worst} ulp"
    assert_close_attn(out_b, out_a, what="c2 fused vs eager-composed")


@pytest.mark.parametrize("p", [0, 1, 7, 15])
def test_fused_cp_step_matches_eager_ops(q3, p):
    """code_predictor.py:40-42 + 58 + 46-47 in one launch; K/V are [B, 8, 16, 128] views of a larger buffer and the
    rotary row is shared by every seat (cp_cos[p])."""
    L, max_bs, B = 2, 80, 61
    g = synth.cpu_gen(60 + p)
    K = synth.randn((L, max_bs, 8, 16, 128), g, 1.0, torch.bfloat16).to(DEV)
    V = synth.randn((L, max_bs, 8, 16, 128), g, 1.0, torch.bfloat16).to(DEV)
    qkv = synth.randn((B, NQ + 2 * NK), g, 1.0, torch.bfloat16).to(DEV)
    qn, kn = (t.to(DEV) for t in norm_weights(61 + p))
    ct, st = rope_tables(16)
    cos, sin = ct[p].to(DEV), st[p].to(DEV)
    Ka, Va = K.clone(), V.clone()
    q, k, v = eager_split(qkv, qn, kn, cos, sin)
    out_a = q3.cp_step(q, k, v, Ka[1, :B], Va[1, :B], p, SCALE)
    out_b = q3.cp_step_qkv(qkv, qn, kn, cos, sin, K[1, :B], V[1, :B], p, SCALE)
    torch.cuda.synchronize()
    assert bits_equal(V, Va), "v slot (raw projection) must be written bit-exactly, nothing else touched"
    n, worst = ulp_flips(K, Ka)
    assert worst <= 1 and n <= max(2, B * 1024 // 200), f"k slot: {n} values differ, up to {worst} ulp"
    assert_close_attn(out_b, out_a, what=f"cp fused vs eager-composed p {p}")
    ref = OA.cp_attention(q.cpu(), Ka[1, :B].cpu(), Va[1, :B].cpu(), p + 1, SCALE)
    assert_close_attn(out_b, ref, what=f"cp fused vs fp32 oracle p {p}")
