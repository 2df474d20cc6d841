"""GPU parity: code-predictor attention (engine/cp_attn.py:33, engine/code_predictor.py:46-47, 58)."""
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


@pytest.mark.parametrize("n_live", list(range(1, 17)))
def test_cp_attn_matches_oracle(q3, n_live):
    d = synth.cp_case(n_live, 64)
    dd = {k: v.to(DEV) for k, v in d.items()}
    poison_allocator((64, 2048))
    out = q3.cp_attn(dd["q"], dd["K"], dd["V"], n_live, SCALE)
    torch.cuda.synchronize()
    ref = OA.cp_attention(d["q"], d["K"], d["V"], n_live, SCALE)
    assert out.shape == (64, 2048)
    assert_close_attn(out, ref, what=f"cp n_live {n_live}")


@pytest.mark.parametrize("p", [0, 1, 7, 14, 15])
def test_cp_step_fused_append(q3, p):
    """Slot-p write is bit-exact and the attention covers slots 0..p, with K/V views whose batch stride exceeds the
    live batch (the reference slices K[l, :B] of a [L, max_bs, 8, 16, 128] buffer, engine/code_predictor.py:56)."""
    L, max_bs, B = 5, 96, 70
    g = synth.cpu_gen(300 + p)
    Kall = synth.randn((L, max_bs, 8, 16, 128), g, 1.0, torch.bfloat16)
    Vall = synth.randn((L, max_bs, 8, 16, 128), g, 1.0, torch.bfloat16)
    q = synth.randn((B, 16, 128), g, 1.0, torch.bfloat16)
    k = synth.randn((B, 8, 128), g, 1.0, torch.bfloat16)
    v = synth.randn((B, 8, 128), g, 1.0, torch.bfloat16)
    l = 3
    rK, rV = Kall[l, :B].clone(), Vall[l, :B].clone()
    ref = OA.cp_step(q, k, v, rK, rV, p, SCALE)
    gK, gV = Kall.to(DEV), Vall.to(DEV)
    poison_allocator((B, 2048))
    out = q3.cp_step(q.to(DEV), k.to(DEV), v.to(DEV), gK[l, :B], gV[l, :B], p, SCALE)
    torch.cuda.synchronize()
    assert_close_attn(out, ref, what=f"cp_step p {p}")
    assert bits_equal(gK[l, :B], rK) and bits_equal(gV[l, :B], rV)
    assert bits_equal(gK[l, B:], Kall[l, B:]) and bits_equal(gK[:l], Kall[:l]), "rows outside the live batch touched"


@pytest.mark.parametrize("layout", ["slot_stride_256", "base_8_byte_aligned"])
def test_cp_attn_strided_fallback(q3, layout):
    """K/V views that a single bulk copy per (seat, head) cannot stage (slot rows not contiguous, or a base that is
    only 8-byte aligned) take the per-lane copy path and give the same results."""
    n_live, B = 11, 48
    d = synth.cp_case(n_live, B)
    if layout == "slot_stride_256":
        Kb = torch.zeros((B, 8, 16, 256), dtype=torch.bfloat16, device=DEV)
        Vb = torch.zeros_like(Kb)
        K, V = Kb[..., :128], Vb[..., :128]
    else:
        Kb = torch.zeros(B * 8 * 16 * 128 + 4, dtype=torch.bfloat16, device=DEV)
        Vb = torch.zeros_like(Kb)
        K, V = Kb[4:].view(B, 8, 16, 128), Vb[4:].view(B, 8, 16, 128)
    K.copy_(d["K"].to(DEV))
    V.copy_(d["V"].to(DEV))
    poison_allocator((B, 2048))
    out = q3.cp_attn(d["q"].to(DEV), K, V, n_live, SCALE)
    torch.cuda.synchronize()
    ref = OA.cp_attention(d["q"], d["K"], d["V"], n_live, SCALE)
    assert_close_attn(out, ref, what=f"cp fallback {layout}")


def test_cp_attn_against_reference_golden(q3, golden_dir):
    """Against CodePredictor._post's attention computed by the reference itself: at the north-star bounds on the
    bf16-rounded inputs the kernel sees, with the input rounding's share added to the max-abs bound on fp32 inputs."""
    g = np.load(os.path.join(golden_dir, "cp_attn.npz"))
    for p in range(16):
        d = synth.cp_case(40 + p, 8, dtype=torch.float32)
        dd = {k: v.to(DEV, torch.bfloat16) for k, v in d.items()}
        out = q3.cp_attn(dd["q"], dd["K"], dd["V"], p + 1, SCALE)
        torch.cuda.synchronize()
        assert_close_attn(out, torch.from_numpy(g[f"p{p}_b16_out"]), what=f"cp golden p {p} (bf16 inputs)")
        assert_close_attn(out, torch.from_numpy(g[f"p{p}_out"]), atol=2e-2, what=f"cp golden p {p} (fp32 inputs)")


def test_cp_full_frame_c4(q3):
    """576 seats, 5 layers, slots 0..15 appended and attended step by step (n_live 1..16),
    compared with the oracle at every (step, layer)."""
    B, L = 576, 5
    g = synth.cpu_gen(44)
    K = torch.zeros(L, B, 8, 16, 128, dtype=torch.bfloat16)
    V = torch.zeros_like(K)
    gK, gV = K.to(DEV), V.to(DEV)
    for p in range(16):
        for l in range(L):
            q = synth.randn((B, 16, 128), g, 1.0, torch.bfloat16)
            k = synth.randn((B, 8, 128), g, 1.0, torch.bfloat16)
            v = synth.randn((B, 8, 128), g, 1.0, torch.bfloat16)
            ref = OA.cp_step(q, k, v, K[l], V[l], p, SCALE)
            out = q3.cp_step(q.to(DEV), k.to(DEV), v.to(DEV), gK[l], gV[l], p, SCALE)
            if l == 0 or p in (0, 15):
                torch.cuda.synchronize()
                assert_close_attn(out, ref, what=f"c4 p {p} l {l}")
    torch.cuda.synchronize()
    assert bits_equal(gK, K) and bits_equal(gV, V)
