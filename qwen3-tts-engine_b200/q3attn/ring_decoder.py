"""The streaming codec decoder's transformer step on the q3attn ring-attention kernel.

Mirrors the transformer part of StreamCore.forward in ring mode (engine/decoder_stream.py:139-181): for a chunk of n
frames of B streams at positions pos .. pos+n-1, each layer normalises, projects q/k/v, applies rotate-half RoPE for the
absolute positions (fp32 angles, cast to the model dtype, decoder_stream.py:141-145), attends through
q3attn.ring_window_attn over the stream's ring of past rotated K/V and the chunk itself (writing the chunk's K/V into
the ring in the same launch, which the reference's caller does after the forward, decoder_stream.py:330-333), and adds
the scaled attention and MLP outputs. The layers are the reference's module objects (duck-typed: input_layernorm,
self_attn.{q,k,v,o}_proj, self_attn_layer_scale.scale, post_attention_layernorm, mlp.{gate,up,down}_proj,
mlp_layer_scale.scale); the rest of the decoder (RVQ, convolutions) is not part of the attention path.
"""
import torch
import torch.nn.functional as F

from . import ops

WIN = 72
PAST = WIN - 1


def _rms(norm, x):
    """decoder_stream.py:129-132."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + norm.variance_epsilon)
    return norm.weight * xf.to(x.dtype)


class RingTransformer:
    def __init__(self, layers, heads: int, head_dim: int, inv_freq: torch.Tensor):
        self.layers, self.H, self.hd, self.L = list(layers), int(heads), int(head_dim), len(layers)
        self.inv_freq = inv_freq.float()
        self.scale = float(head_dim) ** -0.5

    @torch.inference_mode()
    def step(self, h, pos, ring_rows, K, V):
        """h [B, n, D] transformer input of the chunk; pos [B] int64 frames already decoded; ring_rows [B] int64; K / V
        the [S, RING, L, H, hd] fp16 rings (updated in place). Returns the transformer output [B, n, D]."""
        B, n, _ = h.shape
        p = (pos[:, None] + torch.arange(n, device=h.device)[None]).float()
        fr = p[:, :, None] * self.inv_freq[None, None, :].to(h.device)
        emb = torch.cat((fr, fr), dim=-1)
        cos = emb.cos()[:, :, None].to(h.dtype)                  # [B, n, 1, hd]
        sin = emb.sin()[:, :, None].to(h.dtype)
        half = self.hd // 2

        def rot(t):
            return torch.cat((-t[..., half:], t[..., :half]), dim=-1)
        for li, layer in enumerate(self.layers):
            at = layer.self_attn
            r = _rms(layer.input_layernorm, h)
            q = at.q_proj(r).view(B, n, self.H, self.hd)
            k = at.k_proj(r).view(B, n, self.H, self.hd)
            v = at.v_proj(r).view(B, n, self.H, self.hd)
            q = (q * cos + rot(q) * sin).contiguous()
            k = (k * cos + rot(k) * sin).contiguous()
            o = ops.ring_window_attn(q, k, v.contiguous(), K[:, :, li], V[:, :, li], ring_rows, pos, PAST, self.scale,
                                     True)
            h = h + layer.self_attn_layer_scale.scale * at.o_proj(o)
            r = _rms(layer.post_attention_layernorm, h)
            m = layer.mlp
            h = h + layer.mlp_layer_scale.scale * m.down_proj(F.silu(m.gate_proj(r)) * m.up_proj(r))
        return h
