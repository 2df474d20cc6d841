"""Random-init weights in the layout the engine's ``extract()`` produces (engine/model_load.py:37-64).

No checkpoint is available, so the end-to-end frame runs on weights drawn N(0, 0.02) (linear and embedding tables) with
unit norm weights, from a seeded CPU generator so that the GPU engine and the CPU oracle use identical values. RoPE
tables follow the HF rotate-half convention (cos/sin of pos * theta^(-2i/d), duplicated over both halves).
"""
import types

import torch

SIZES = {
    # talker hidden, ffn, layers, heads, kv heads, head_dim, vocab (codec_head rows), cp hidden, cp ffn, cp layers
    "0.6B": dict(H=1024, ffn=3072, n_layers=28, cp_H=1024, cp_ffn=3072, cp_layers=5),
    "1.7B": dict(H=2048, ffn=6144, n_layers=28, cp_H=1024, cp_ffn=3072, cp_layers=5),
}
HEADS, KV_HEADS, HEAD_DIM = 16, 8, 128
VOCAB, CP_VOCAB, N_GROUPS = 3072, 2048, 16
EOS = 2150                        # a codec special id above the 2048 audio codes (only ids >= vocab-1024 are specials)
ROPE_THETA = 1_000_000.0


def rope_tables(n_pos: int, dim: int = HEAD_DIM, theta: float = ROPE_THETA):
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    f = torch.arange(n_pos, dtype=torch.float64)[:, None] * inv[None, :]
    emb = torch.cat([f, f], -1)
    return emb.cos().float(), emb.sin().float()


def _layer(g, H, ffn, std):
    nq, nk = HEADS * HEAD_DIM, KV_HEADS * HEAD_DIM
    r = lambda *s: torch.randn(*s, generator=g) * std
    return types.SimpleNamespace(
        ln1=torch.ones(H), ln2=torch.ones(H),
        qkv=r(nq + 2 * nk, H), qn=torch.ones(HEAD_DIM), kn=torch.ones(HEAD_DIM),
        o=r(H, nq), gu=r(2 * ffn, H), down=r(H, ffn))


def random_weights(seed: int = 0, size: str = "0.6B", max_pos: int = 4096, std: float = 0.02, n_layers=None):
    """fp32 CPU weights in the extract() layout; cast with :func:`cast`. ``n_layers`` shortens the talker for tests."""
    c = SIZES[size]
    g = torch.Generator().manual_seed(int(seed))
    H, cpH = c["H"], c["cp_H"]
    nl = c["n_layers"] if n_layers is None else n_layers
    W = types.SimpleNamespace(size=size, H=H, n_layers=nl, heads=HEADS, kv_heads=KV_HEADS, head_dim=HEAD_DIM, ffn=c["ffn"],
                              vocab=VOCAB, eos=EOS, n_groups=N_GROUPS, device=torch.device("cpu"), dtype=torch.float32)
    W.layers = [_layer(g, H, c["ffn"], std) for _ in range(nl)]
    W.norm = torch.ones(H)
    W.codec_emb = torch.randn(VOCAB, H, generator=g) * std
    W.codec_head = torch.randn(VOCAB, H, generator=g) * std
    W.cos, W.sin = rope_tables(max_pos)
    W.cp_H, W.cp_ffn, W.cp_vocab = cpH, c["cp_ffn"], CP_VOCAB
    W.cp_layers = [_layer(g, cpH, c["cp_ffn"], std) for _ in range(c["cp_layers"])]
    W.cp_norm = torch.ones(cpH)
    W.cp_emb = torch.randn(N_GROUPS - 1, CP_VOCAB, H, generator=g) * std
    W.cp_head = torch.randn(N_GROUPS - 1, CP_VOCAB, cpH, generator=g) * std
    if H != cpH:
        W.cp_proj_w = torch.randn(cpH, H, generator=g) * std
        W.cp_proj_b = torch.zeros(cpH)
    else:
        W.cp_proj_w = W.cp_proj_b = None
    W.cp_cos, W.cp_sin = rope_tables(16)
    return W


def cast(W, dtype, device="cpu"):
    """Copy of W with every tensor cast to ``dtype`` on ``device`` (a bf16 round trip for the oracle: cast(cast(W,
    bf16), fp32) holds exactly the values the bf16 engine computes with)."""
    def cv(x):
        return x.to(device=device, dtype=dtype).contiguous() if torch.is_tensor(x) else x
    out = types.SimpleNamespace(**{k: cv(v) for k, v in vars(W).items()})
    out.layers = [types.SimpleNamespace(**{k: cv(v) for k, v in vars(l).items()}) for l in W.layers]
    out.cp_layers = [types.SimpleNamespace(**{k: cv(v) for k, v in vars(l).items()}) for l in W.cp_layers]
    out.device, out.dtype = torch.device(device), dtype
    return out
