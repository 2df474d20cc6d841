"""fp32 CPU restatement of one engine frame step (test infrastructure only; see oracle/__init__.py).

Restates, with greedy sampling (top_k = 1):
  ops.rms / rope / mlp / sample_topk             engine/ops.py:51-76
  Talker._decode, _cb0_logits, _tail, _frame     engine/talker.py:63-80, 90-112
  CodePredictor._pre/_post/_s/run                engine/code_predictor.py:37-72
The talker's K/V live in a paged pool addressed through a block table (any page size, any table); the attention is
oracle.attention.decode_attention, i.e. Talker._attn_ref over the gathered pages.
"""
import torch
import torch.nn.functional as F

from .attention import append_paged, decode_attention

NEG = float("-inf")


def rms(x, w, eps: float = 1e-6):
    """engine/ops.py:51-55: normalise in fp32, cast back to x's dtype, then scale."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * xf.to(x.dtype)


def rope(x, cos, sin):
    """engine/ops.py:58-60: rotate-half RoPE."""
    h = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., h:], x[..., :h]), dim=-1) * sin


def mlp(x, w, ffn: int):
    """engine/ops.py:63-65: SiLU-gated MLP with the concatenated gate/up projection."""
    gu = F.linear(x, w.gu)
    return F.linear(F.silu(gu[..., :ffn]) * gu[..., ffn:], w.down)


def greedy(logits):
    """engine/ops.py:68-76 with k = 1: the single top-k value has softmax weight 1, so the multinomial draw always picks
    it; the sample is ``topk(logits, 1).indices``."""
    return torch.topk(logits, 1, dim=-1).indices[:, 0]


class CodePredictorOracle:
    """engine/code_predictor.py:14-72 in fp32 with a static 16-slot K/V scratch per layer."""

    def __init__(self, W, max_bs):
        self.W, self.L = W, len(W.cp_layers)
        self.nh, self.nkv, self.hd = 16, 8, W.head_dim
        self.scale = float(W.head_dim) ** -0.5
        self.ffn = W.cp_ffn
        self.K = torch.zeros(self.L, max_bs, self.nkv, 16, self.hd)
        self.V = torch.zeros(self.L, max_bs, self.nkv, 16, self.hd)
        self.mask = torch.full((16, 16), NEG).triu(1)

    def proj(self, x):
        return x if self.W.cp_proj_w is None else F.linear(x, self.W.cp_proj_w, self.W.cp_proj_b)

    def _s(self, x, B, p):
        W = self.W
        nq, nk = self.nh * self.hd, self.nkv * self.hd
        cos, sin = W.cp_cos[p], W.cp_sin[p]
        for l in range(self.L):
            w = W.cp_layers[l]
            K, V = self.K[l, :B], self.V[l, :B]
            qkv = F.linear(rms(x, w.ln1), w.qkv)                                      # code_predictor.py:39-42
            q = rope(rms(qkv[:, :nq].view(B, self.nh, self.hd), w.qn), cos, sin)
            k = rope(rms(qkv[:, nq:nq + nk].view(B, self.nkv, self.hd), w.kn), cos, sin)
            v = qkv[:, nq + nk:].view(B, self.nkv, self.hd)
            K[:, :, p] = k                                                            # code_predictor.py:58
            V[:, :, p] = v
            att = torch.matmul(q.view(B, self.nkv, self.nh // self.nkv, self.hd), K.transpose(-1, -2)) * self.scale + self.mask[p]
            o = torch.matmul(torch.softmax(att, dim=-1), V).reshape(B, nq)            # code_predictor.py:46-47
            x = x + F.linear(o, w.o)
            gu = F.linear(rms(x, w.ln2), w.gu)
            x = x + F.linear(F.silu(gu[..., :self.ffn]) * gu[..., self.ffn:], w.down)
        return rms(x, W.cp_norm)

    def run(self, h, c0):
        """code_predictor.py:62-72: slot 0 from the talker hidden, then 15 greedy steps."""
        W = self.W
        B = h.shape[0]
        self._s(self.proj(h), B, 0)
        e = W.codec_emb[c0]
        embs, codes = [e], []
        for i in range(15):
            hid = self._s(self.proj(e), B, i + 1)
            c = greedy(F.linear(hid, W.cp_head[i]).float())
            codes.append(c)
            e = W.cp_emb[i][c]
            embs.append(e)
        return torch.stack(codes, 1), torch.stack(embs, 1).sum(1)


class FrameOracle:
    """Seats with paged K/V and the per-seat sampling state of engine/talker.py:29-47, fp32 on the CPU.

    ``block_table`` has n_seats + 1 rows (the last is the scratch seat that padded rows point at, talker.py:29)."""

    def __init__(self, W, n_seats, block_table, page, num_pages, max_bs, rep_penalty=1.05, min_new=2, max_text=16):
        self.W = W
        self.n_seats, self.page = n_seats, page
        self.nh, self.nkv, self.hd, self.H, self.ffn = W.heads, W.kv_heads, W.head_dim, W.H, W.ffn
        self.scale = float(self.hd) ** -0.5
        self.rep, self.min_new = rep_penalty, min_new
        S1 = n_seats + 1
        self.bt = block_table
        self.kc = [torch.zeros(num_pages, page, self.nkv, self.hd) for _ in W.layers]
        self.vc = [torch.zeros(num_pages, page, self.nkv, self.hd) for _ in W.layers]
        self.pos = torch.zeros(S1, dtype=torch.int64)
        self.x_in = torch.zeros(S1, self.H)
        self.seen = torch.zeros(S1, W.vocab, dtype=torch.bool)
        self.ngen = torch.zeros(S1, dtype=torch.int64)
        self.trail = torch.zeros(S1, max_text + 1, self.H)
        self.trail_len = torch.zeros(S1, dtype=torch.int64)
        sup = torch.zeros(W.vocab)
        sup[W.vocab - 1024:] = NEG
        sup[W.eos] = 0.0
        self.suppress = sup                                                  # talker.py:43
        self.eos_col = torch.zeros(W.vocab, dtype=torch.bool)
        self.eos_col[W.eos] = True
        self.cp = CodePredictorOracle(W, max_bs)

    def decode(self, x, seat, pos):
        """talker.py:63-80 with the append placed through the block table and the attention over ctx = pos + 1."""
        W = self.W
        B = x.shape[0]
        nq, nk = self.nh * self.hd, self.nkv * self.hd
        cos, sin = W.cos[pos][:, None, :], W.sin[pos][:, None, :]
        bt = self.bt[seat]
        for l in range(len(W.layers)):
            w = W.layers[l]
            qkv = F.linear(rms(x, w.ln1), w.qkv)
            q = rope(rms(qkv[:, :nq].view(B, self.nh, self.hd), w.qn), cos, sin)
            k = rope(rms(qkv[:, nq:nq + nk].view(B, self.nkv, self.hd), w.kn), cos, sin)
            v = qkv[:, nq + nk:].view(B, self.nkv, self.hd)
            append_paged(self.kc[l], self.vc[l], k, v, pos, bt)
            o = decode_attention(q, self.kc[l], self.vc[l], pos + 1, bt, self.scale)
            x = x + F.linear(o.reshape(B, nq), w.o)
            x = x + mlp(rms(x, w.ln2), w, self.ffn)
        return rms(x, W.norm)

    def cb0_logits(self, h, seat):
        """talker.py:90-94."""
        lg = F.linear(h, self.W.codec_head).float()
        lg = torch.where(self.seen[seat], torch.where(lg < 0, lg * self.rep, lg / self.rep), lg) + self.suppress
        return lg.masked_fill((self.ngen[seat] < self.min_new)[:, None] & self.eos_col[None, :], NEG)

    def tail(self, h, seat):
        """talker.py:96-105 with greedy sampling."""
        c0 = greedy(self.cb0_logits(h, seat))
        g = self.ngen[seat].clone()
        self.seen[seat, c0] = True
        self.ngen[seat] = g + 1
        codes, acc = self.cp.run(h, c0)
        t = self.trail[seat, torch.minimum(g, self.trail_len[seat])]
        self.x_in[seat] = acc + t
        return torch.cat([c0[:, None], codes], 1)

    def frame(self, seat):
        """talker.py:107-112 for the seat rows ``seat`` (padded rows carry the scratch seat id n_seats)."""
        pos = self.pos[seat].clone()
        h = self.decode(self.x_in[seat], seat, pos)
        self.pos[seat] = torch.where(seat == self.n_seats, torch.zeros_like(pos), pos + 1)
        return self.tail(h, seat)
