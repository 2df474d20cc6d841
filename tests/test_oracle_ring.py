"""CPU: the ring-attention oracle (oracle/ring.py) inside a CPU twin of the decoder transformer step reproduces what
the reference's own StreamDecoder._step / StreamCore.forward computed on the same small decoder
(tests/golden/ring.npz, engine/decoder_stream.py:134-181, 325-339): the oracle is pinned to the reference."""
import os

import numpy as np
import torch
import torch.nn.functional as F

import make_golden as mg
from oracle import ring as OR

RING, PAST = 88, 71


def _rms(w, eps, x):
    xf = x.float()
    return w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


@torch.inference_mode()
def test_oracle_ring_attention_reproduces_the_reference_stream(golden_dir):
    c = mg.RING_CASE
    gold = np.load(os.path.join(golden_dir, "ring.npz"))
    D, H, hd, L, S = c["D"], c["H"], c["hd"], c["L"], c["S"]
    layers, inv_freq = mg.ring_model(c["seed"], D, H, hd, L)
    K = torch.zeros(S + 1, RING, L, H, hd)
    V = torch.zeros_like(K)
    pos = torch.zeros(S + 1, dtype=torch.int64)
    for call, (seats, n) in enumerate(c["calls"]):
        rows = torch.tensor(seats)
        B = len(seats)
        h = mg.ring_h(call, B, n, D, c["seed"])
        p = (pos[rows][:, None] + torch.arange(n)[None]).float()
        fr = p[:, :, None] * inv_freq[None, None, :]
        emb = torch.cat((fr, fr), -1)
        cos, sin = emb.cos()[:, :, None], emb.sin()[:, :, None]

        def rot(t):
            return torch.cat((-t[..., hd // 2:], t[..., :hd // 2]), -1)
        newk, newv = [], []
        for li, layer in enumerate(layers):
            at = layer.self_attn
            r = _rms(layer.input_layernorm.weight, 1e-5, h)
            q = at.q_proj(r).view(B, n, H, hd)
            k = at.k_proj(r).view(B, n, H, hd)
            v = at.v_proj(r).view(B, n, H, hd)
            q, k = q * cos + rot(q) * sin, k * cos + rot(k) * sin
            o = OR.ring_attention(q, k, v, K[rows, :, li], V[rows, :, li], pos[rows], PAST, hd ** -0.5)
            h = h + layer.self_attn_layer_scale.scale * at.o_proj(o)
            r = _rms(layer.post_attention_layernorm.weight, 1e-5, h)
            m = layer.mlp
            h = h + layer.mlp_layer_scale.scale * m.down_proj(F.silu(m.gate_proj(r)) * m.up_proj(r))
            newk.append(k)
            newv.append(v)
        ref = torch.from_numpy(gold[f"h{call}"].astype(np.float32))
        got = _rms(torch.ones(D), 1e-5, h)
        assert float((got - ref).abs().max()) < 1e-2, f"call {call}"      # fp16-stored fixture, fp32 maths
        for li in range(L):                                                 # the caller's ring write
            for j in range(n):
                K[rows, (pos[rows] + j) % RING, li] = newk[li][:, j]
                V[rows, (pos[rows] + j) % RING, li] = newv[li][:, j]
        pos[rows] += n
    assert np.array_equal(pos.numpy(), gold["pos"])
    assert float((K[:S, :, L - 1] - torch.from_numpy(gold["K_last"].astype(np.float32))).abs().max()) < 1e-2
