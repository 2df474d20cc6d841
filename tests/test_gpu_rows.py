"""GPU parity: the row kernels around the attention layers against the reference's own ops (engine/ops.py:51-65,
restated in oracle.frame) run eagerly in bf16 on the same GPU: residual add + RMSNorm, the SiLU gate, and the in-place
q/k RMSNorm + RoPE of QKV rows. Equal except for rare one-ulp flips (a different fp32 summation order of the squares,
expf against torch's exp)."""
import pytest
import torch
import torch.nn.functional as F

from helpers import bits_equal
from oracle import frame as OF
from q3attn import synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def q3():
    import q3attn
    q3attn._lib.load()
    return q3attn


def ulp_flips(a, b):
    ai = a.contiguous().view(torch.int16).to(torch.int32)
    bi = b.contiguous().view(torch.int16).to(torch.int32)
    d = (ai - bi).abs()
    return int((d != 0).sum()), int(d.max())


def assert_near_exact(got, ref, what, frac=5e-3):
    n, worst = ulp_flips(got, ref)
    assert worst <= 1 and n <= max(2, int(frac * ref.numel())), f"{what}: {n} values differ, up to {worst} ulp"


@pytest.mark.parametrize("H", [1024, 2048])
@pytest.mark.parametrize("with_residual", [False, True])
def test_add_rms_norm(q3, H, with_residual):
    g = synth.cpu_gen(H + with_residual)
    rows = 333
    x = synth.randn((rows, H), g, 1.5, torch.bfloat16).to(DEV)
    r = synth.randn((rows, H), g, 0.7, torch.bfloat16).to(DEV) if with_residual else None
    w = (1 + 0.1 * synth.randn((H,), g)).to(torch.bfloat16).to(DEV)
    x_ref = x + r if with_residual else x.clone()
    y_ref = OF.rms(x_ref, w)
    y = q3.add_rms_norm(x, w, r)
    torch.cuda.synchronize()
    assert bits_equal(x, x_ref), "the residual stream must hold bf16(x + r) exactly"
    assert_near_exact(y, y_ref, f"rms H {H}")


def test_silu_mul(q3):
    g = synth.cpu_gen(3)
    F_ = 3072
    gu = synth.randn((300, 2 * F_), g, 2.0, torch.bfloat16).to(DEV)
    ref = F.silu(gu[:, :F_]) * gu[:, F_:]
    out = q3.silu_mul(gu)
    torch.cuda.synchronize()
    assert_near_exact(out, ref, "silu * u")


@pytest.mark.parametrize("shared_row", [False, True])
def test_qk_norm_rope_in_place(q3, shared_row):
    g = synth.cpu_gen(5 + shared_row)
    T = 97
    qkv = synth.randn((T, 4096), g, 1.0, torch.bfloat16).to(DEV)
    qn = (1 + 0.1 * synth.randn((128,), g)).to(torch.bfloat16).to(DEV)
    kn = (1 + 0.1 * synth.randn((128,), g)).to(torch.bfloat16).to(DEV)
    ang = torch.arange(T)[:, None] * (1e6 ** (-torch.arange(0, 128, 2) / 128))[None]
    cos = torch.cat([ang, ang], -1).cos().to(torch.bfloat16).to(DEV)
    sin = torch.cat([ang, ang], -1).sin().to(torch.bfloat16).to(DEV)
    if shared_row:
        cos, sin = cos[7], sin[7]
    c = cos.view(-1, 1, 128)
    s = sin.view(-1, 1, 128)
    q_ref = OF.rope(OF.rms(qkv[:, :2048].view(T, 16, 128), qn), c, s)
    k_ref = OF.rope(OF.rms(qkv[:, 2048:3072].view(T, 8, 128), kn), c, s)
    v_ref = qkv[:, 3072:].clone()
    q3.qk_norm_rope_(qkv, qn, kn, cos, sin)
    torch.cuda.synchronize()
    assert_near_exact(qkv[:, :2048].reshape(T, 16, 128), q_ref, "q")
    assert_near_exact(qkv[:, 2048:3072].reshape(T, 8, 128), k_ref, "k")
    assert bits_equal(qkv[:, 3072:], v_ref)
