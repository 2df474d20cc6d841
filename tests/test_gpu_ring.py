"""GPU parity: the streaming codec decoder's windowed ring attention (engine/decoder_stream.py:147-181).

* the kernel against the oracle restatement with the reference's fp16 rounding points, on random rings and positions
  around every window and ring edge, plus the ring write (the chunk's K/V in slots (pos + j) % RING, nothing else
  touched);
* the decoder transformer step (q3attn.ring_decoder) against what the reference's own StreamDecoder._step /
  StreamCore.forward computed in fp32 on a small decoder, over 26 chunks that wrap the 88-slot ring
  (tests/golden/ring.npz)."""
import os
import types

import numpy as np
import pytest
import torch

import make_golden as mg
from helpers import bits_equal
from oracle import ring as OR
from q3attn import synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
RING, PAST = 88, 71


@pytest.fixture(scope="module")
def q3():
    import q3attn
    q3attn._lib.load()
    return q3attn


# (one-frame kernel, multi-frame kernel) pairs; together they cover every selection of both
RING_KERNELS = [(6, 1), (2, 1), (1, 1), (0, 0), (3, 2), (4, 3), (5, 4)]


@pytest.fixture(params=RING_KERNELS, autouse=True,
                ids=["default", "heads", "cta_per_head", "mma_heads", "mma_narrow", "mma_one", "tma_pipe"])
def ring_kernels(q3, request):
    """Every test runs on each kernel selection (one-frame kernel, multi-frame kernel). One frame: 6 = nothing staged,
    4 / 8 warps per (stream, head) of 64 / 128 dims loading straight into registers (default); 2 = scalar math, one
    warp per head, 4 x 64 / 2 x 128 heads per CTA; 1 = one CTA per (stream, head); 0 / 3 / 4 = tensor cores with
    4 / 2 / 1 heads of 64 per CTA; 5 = the persistent TMA pipeline (head_dim 64). Chunks of 2 .. 16 frames: 1 = one
    CTA per (stream, head) (default, also for 17 frames); 0 / 2 / 3 = tensor cores, one warp per head, with 2 / 4 / 1
    heads of 64 per CTA; 4 = the persistent TMA pipeline (2 .. 8 frames, head_dim 64). Calls a selection does not fit
    fall back to one CTA per (stream, head)."""
    frame, chunk = request.param
    prev_f = q3.set_ring_frame_kernel(frame)
    prev_c = q3.set_ring_chunk_kernel(chunk)
    yield request.param
    q3.set_ring_frame_kernel(prev_f)
    q3.set_ring_chunk_kernel(prev_c)


@pytest.mark.parametrize("hd,H", [(64, 8), (128, 4), (64, 6), (128, 3)])
@pytest.mark.parametrize("n", [1, 2, 4, 8, 16, 17])
def test_ring_attention_matches_oracle(q3, hd, H, n):
    g = synth.cpu_gen(hd + n)
    pos = torch.tensor([0, 1, 5, 70, 71, 72, 87, 88, 150, 1000], dtype=torch.int64)
    B, S, L, li = len(pos), 12, 2, 1
    rows = torch.randperm(S, generator=g)[:B]
    K = synth.randn((S, RING, L, H, hd), g, 1.0, torch.float16)
    V = synth.randn((S, RING, L, H, hd), g, 1.0, torch.float16)
    q = synth.randn((B, n, H, hd), g, 1.0, torch.float16)
    k = synth.randn((B, n, H, hd), g, 1.0, torch.float16)
    v = synth.randn((B, n, H, hd), g, 1.0, torch.float16)
    Kg, Vg = K.to(DEV), V.to(DEV)
    out = q3.ring_window_attn(q.to(DEV), k.to(DEV), v.to(DEV), Kg[:, :, li], Vg[:, :, li], rows.to(DEV), pos.to(DEV),
                              PAST, hd ** -0.5, True)
    torch.cuda.synchronize()
    ref = OR.ring_attention(q, k, v, K[rows, :, li], V[rows, :, li], pos, PAST, hd ** -0.5, emulate_fp16=True)
    err = (out.float().cpu() - ref).abs()
    assert float(err.max()) <= 1e-2 + 2e-2 * float(ref.abs().max()), f"max err {float(err.max()):.3e}"
    # ring write: slots (pos + j) % RING of layer li get the chunk's rows, everything else is untouched
    K2, V2 = K.clone(), V.clone()
    for b in range(B):
        for j in range(n):
            K2[rows[b], (pos[b] + j) % RING, li] = k[b, j]
            V2[rows[b], (pos[b] + j) % RING, li] = v[b, j]
    assert bits_equal(Kg, K2) and bits_equal(Vg, V2)


@pytest.mark.parametrize("n", [1, 4])
def test_ring_attention_far_positions(q3, n):
    """Positions far past 2^31 (a stream's frame counter is int64): the slot arithmetic stays exact."""
    hd, H = 64, 8
    g = synth.cpu_gen(900 + n)
    pos = torch.tensor([2**31 - 2, 2**31 - 1, 2**31, 2**31 + 87, 2**32 + 5, 2**40 + 13, 2**62 + 71, 2**63 - 64],
                       dtype=torch.int64)
    B, S = len(pos), 10
    rows = torch.randperm(S, generator=g)[:B]
    K = synth.randn((S, RING, H, hd), g, 1.0, torch.float16)
    V = synth.randn((S, RING, H, hd), g, 1.0, torch.float16)
    q = synth.randn((B, n, H, hd), g, 1.0, torch.float16)
    k = synth.randn((B, n, H, hd), g, 1.0, torch.float16)
    v = synth.randn((B, n, H, hd), g, 1.0, torch.float16)
    Kg, Vg = K.to(DEV), V.to(DEV)
    out = q3.ring_window_attn(q.to(DEV), k.to(DEV), v.to(DEV), Kg, Vg, rows.to(DEV), pos.to(DEV), PAST, hd ** -0.5,
                              True)
    torch.cuda.synchronize()
    ref = OR.ring_attention(q, k, v, K[rows], V[rows], pos, PAST, hd ** -0.5, emulate_fp16=True)
    err = (out.float().cpu() - ref).abs()
    assert float(err.max()) <= 1e-2 + 2e-2 * float(ref.abs().max()), f"max err {float(err.max()):.3e}"
    K2, V2 = K.clone(), V.clone()
    for b in range(B):
        for j in range(n):
            K2[rows[b], (int(pos[b]) + j) % RING] = k[b, j]
            V2[rows[b], (int(pos[b]) + j) % RING] = v[b, j]
    assert bits_equal(Kg, K2) and bits_equal(Vg, V2)


def test_decoder_transformer_matches_reference_stream(q3, golden_dir):
    from q3attn.ring_decoder import RingTransformer, _rms
    c = mg.RING_CASE
    gold = np.load(os.path.join(golden_dir, "ring.npz"))
    D, H, hd, L, S = c["D"], c["H"], c["hd"], c["L"], c["S"]
    layers, inv_freq = mg.ring_model(c["seed"], D, H, hd, L)
    assert str(gold["digest"]) == mg.digest(layers[0].self_attn.q_proj.weight, mg.ring_h(0, 3, 4, D, c["seed"]))

    def dev(x):
        if isinstance(x, torch.nn.Module):
            return x.to(DEV, torch.float16)
        if torch.is_tensor(x):
            return x.to(DEV, torch.float16)
        if isinstance(x, types.SimpleNamespace):
            return types.SimpleNamespace(**{k: dev(v) for k, v in vars(x).items()})
        return x
    T = RingTransformer([dev(l) for l in layers], H, hd, inv_freq)
    K = torch.zeros(S + 1, RING, L, H, hd, dtype=torch.float16, device=DEV)
    V = torch.zeros_like(K)
    pos = torch.zeros(S + 1, dtype=torch.int64, device=DEV)
    norm = types.SimpleNamespace(weight=torch.ones(D, dtype=torch.float16, device=DEV), variance_epsilon=1e-5)
    worst = 0.0
    for call, (seats, n) in enumerate(c["calls"]):
        rows = torch.tensor(seats, dtype=torch.int64, device=DEV)
        h = mg.ring_h(call, len(seats), n, D, c["seed"]).to(DEV, torch.float16)
        out = _rms(norm, T.step(h, pos[rows].contiguous(), rows, K, V)).float().cpu()
        ref = torch.from_numpy(gold[f"h{call}"].astype(np.float32))
        rel = float((out - ref).norm() / ref.norm())
        worst = max(worst, rel)
        assert rel < 2e-2, f"call {call}: transformer output relative error {rel:.3e}"
        pos[rows] += n
    torch.cuda.synchronize()
    assert np.array_equal(pos.cpu().numpy(), gold["pos"])
    for name, ring in (("K_last", K), ("V_last", V)):
        got = ring[:S, :, L - 1].float().cpu()
        ref = torch.from_numpy(gold[name].astype(np.float32))
        rel = float((got - ref).norm() / ref.norm())
        assert rel < 2e-2, f"{name}: relative error {rel:.3e}"


@pytest.mark.parametrize("hd,H", [(64, 8), (128, 4)])
@pytest.mark.parametrize("n", [1, 4, 8, 16])
def test_ring_slots_no_query_sees_are_never_used(q3, hd, H, n):
    """Ring slots outside every query's window (never written yet, or older than the window) may hold anything, NaN
    included: the outputs equal those computed with the same slots zeroed."""
    g = synth.cpu_gen(500 + hd + n)
    pos = torch.tensor([0, 1, 3, 40, 71, 72, 90, 500], dtype=torch.int64)
    B, S = len(pos), 9
    rows = torch.arange(B)
    K = synth.randn((S, RING, H, hd), g, 1.0, torch.float16)
    V = synth.randn((S, RING, H, hd), g, 1.0, torch.float16)
    for b in range(B):
        p = int(pos[b])
        for j in range(RING):
            d = ((p - 1) - j) % RING
            if d > min(p - 1, PAST - 1):
                K[b, j] = float("nan")
                V[b, j] = float("inf") if j % 2 else float("nan")
    Kz, Vz = torch.nan_to_num(K, nan=0.0, posinf=0.0), torch.nan_to_num(V, nan=0.0, posinf=0.0)
    q = synth.randn((B, n, H, hd), g, 1.0, torch.float16)
    k = synth.randn((B, n, H, hd), g, 1.0, torch.float16)
    v = synth.randn((B, n, H, hd), g, 1.0, torch.float16)
    outs = []
    for KK, VV in ((K, V), (Kz, Vz)):
        outs.append(q3.ring_window_attn(q.to(DEV), k.to(DEV), v.to(DEV), KK.to(DEV), VV.to(DEV), rows.to(DEV),
                                        pos.to(DEV), PAST, hd ** -0.5, False))
    torch.cuda.synchronize()
    assert torch.isfinite(outs[0]).all()
    assert bits_equal(outs[0], outs[1])
