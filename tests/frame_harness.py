"""Test and benchmark harness: the engine's frame step on the GPU with every attention and K/V append on the q3attn
kernels. It is test infrastructure, not part of the q3attn package: it restates the reference engine's own host
orchestration so the kernels can be checked and timed inside the frame they serve.

Mirrors engine/talker.py (Talker: seats, paged K/V, per-seat sampling state, one CUDA graph per batch bucket) and
engine/code_predictor.py (CodePredictor: 16-slot K/V scratch, 15 sampled steps), with the attention hot path replaced:
  talker layer  (talker.py:69-77)   q/k RMSNorm + RoPE, K/V append and paged decode in one launch
                                    (q3attn.paged_decode_qkv, straight from the QKV projection)
  CP layer      (code_predictor.py:40-42, 58, 46-47)  q/k RMSNorm + RoPE, slot-p write and attention in one launch
                                    (q3attn.cp_step_qkv)
GEMMs, the layer norms, the MLP and sampling stay PyTorch ops in the reference's order and dtype (engine/ops.py:40-76).

Differences from the reference, all in layout, none in the maths: the K/V pools are paged with a configurable page
size and block table (default 16-token pages; the reference uses 256-token pages and the identity table,
talker.py:25, 42), and the weights come from q3attn.weights (random init; no checkpoint in this build).
"""
import torch
import torch.nn.functional as F

from q3attn import ops

NEG = float("-inf")


def rms(x, w, eps: float = 1e-6):
    """engine/ops.py:51-55."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * xf.to(x.dtype)


def rope(x, cos, sin):
    """engine/ops.py:58-60."""
    h = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., h:], x[..., :h]), dim=-1) * sin


def _split_qkv(qkv, w, cos, sin, B, nh, nkv, hd):
    """q, k, v of one layer with the norms and RoPE as PyTorch ops (engine/talker.py:69-71,
    engine/code_predictor.py:40-42); k and v come back with one shared row stride."""
    nq, nk = nh * hd, nkv * hd
    q = rope(rms(qkv[:, :nq].view(B, nh, hd), w.qn), cos, sin)
    k = rope(rms(qkv[:, nq:nq + nk].view(B, nkv, hd), w.kn), cos, sin)
    v = qkv[:, nq + nk:].contiguous().view(B, nkv, hd)
    return q, k.contiguous(), v


def mlp(x, w, ffn: int):
    """engine/ops.py:63-65."""
    gu = F.linear(x, w.gu)
    return F.linear(F.silu(gu[..., :ffn]) * gu[..., ffn:], w.down)


def sample_topk(logits, temperature: float, k: int, gen):
    """engine/ops.py:68-76: temperature warp, keep the k largest, sample (k = 1 is greedy)."""
    vals, idx = torch.topk(logits, k, dim=-1)
    p = torch.softmax(vals / temperature, dim=-1)
    j = torch.multinomial(p, 1, generator=gen)
    return idx.gather(1, j).squeeze(1)


class CodePredictor:
    """engine/code_predictor.py:14-72 with the attention and slot write of each (step, layer) in one q3attn.cp_step."""

    def __init__(self, W, max_bs, temperature=0.9, top_k=50, fuse_qk_norm_rope=True, fused_sampler=True):
        self.W, self.L = W, len(W.cp_layers)
        self.fuse = fuse_qk_norm_rope
        self.fused_sampler = fused_sampler
        self.nh, self.nkv, self.hd = 16, 8, W.head_dim
        self.ffn, self.scale = W.cp_ffn, float(W.head_dim) ** -0.5
        self.temperature, self.top_k = temperature, top_k
        d, dt = W.device, W.dtype
        self.K = torch.zeros(self.L, max_bs, self.nkv, 16, self.hd, dtype=dt, device=d)
        self.V = torch.zeros(self.L, max_bs, self.nkv, 16, self.hd, dtype=dt, device=d)

    def proj(self, x):
        return x if self.W.cp_proj_w is None else F.linear(x, self.W.cp_proj_w, self.W.cp_proj_b)

    def _s(self, x, B, p):
        W = self.W
        cos, sin = W.cp_cos[p], W.cp_sin[p]
        if self.fuse:
            # code_predictor.py:37-50 with the q3attn row kernels: residual add + RMSNorm and the SiLU gate in one
            # launch each, q/k norm + RoPE + slot write + attention in one (the residual stream is updated in place)
            x = x.clone()
            r = None
            for l in range(self.L):
                w = W.cp_layers[l]
                qkv = F.linear(ops.add_rms_norm(x, w.ln1, r), w.qkv)
                o = ops.cp_step_qkv(qkv, w.qn, w.kn, cos, sin, self.K[l, :B], self.V[l, :B], p, self.scale)
                h = ops.add_rms_norm(x, w.ln2, F.linear(o, w.o))
                r = F.linear(ops.silu_mul(F.linear(h, w.gu)), w.down)
            return ops.add_rms_norm(x, W.cp_norm, r)
        for l in range(self.L):   # the same maths as separate PyTorch ops
            w = W.cp_layers[l]
            qkv = F.linear(rms(x, w.ln1), w.qkv)                                        # code_predictor.py:39
            q, k, v = _split_qkv(qkv, w, cos, sin, B, self.nh, self.nkv, self.hd)     # :40-42
            o = ops.cp_step(q, k, v, self.K[l, :B], self.V[l, :B], p, self.scale)    # :58, 46-47
            x = x + F.linear(o, w.o)
            gu = F.linear(rms(x, w.ln2), w.gu)
            x = x + F.linear(F.silu(gu[..., :self.ffn]) * gu[..., self.ffn:], w.down)
        return rms(x, W.cp_norm)

    def run(self, h, c0, gen, e0=None):
        """code_predictor.py:62-72. gen: the talker's SamplerRng (fused sampler) or torch.Generator; e0: codec_emb[c0]
        when the caller already has it."""
        W = self.W
        B = h.shape[0]
        self._s(self.proj(h), B, 0)
        e = W.codec_emb[c0] if e0 is None else e0
        embs, codes = [e], []
        for i in range(15):
            hid = self._s(self.proj(e), B, i + 1)
            if self.fused_sampler:   # top-k draw + cp_emb[i][c] in one launch (code_predictor.py:70-71)
                c, e = ops.sample_topk(F.linear(hid, W.cp_head[i]), self.temperature, self.top_k, gen,
                                       emb=W.cp_emb[i])
            else:
                c = sample_topk(F.linear(hid, W.cp_head[i]).float(), self.temperature, self.top_k, gen)
                e = W.cp_emb[i][c]
            codes.append(c)
            embs.append(e)
        return torch.stack(codes, 1), torch.stack(embs, 1).sum(1)

    def tf_logits(self, h, codes16):
        """code_predictor.py:74-82: the 15 logits [B,15,2048] (fp32) given the frame's 16 codes (teacher-forced)."""
        W = self.W
        B = h.shape[0]
        self._s(self.proj(h), B, 0)
        e = W.codec_emb[codes16[:, 0]]
        out = []
        for i in range(15):
            hid = self._s(self.proj(e), B, i + 1)
            out.append(F.linear(hid, W.cp_head[i]).float())
            e = W.cp_emb[i][codes16[:, i + 1]]
        return torch.stack(out, 1)


class Talker:
    """engine/talker.py:20-138 over paged K/V pools and the q3attn kernels.

    block_table: int32 [n_seats + 1, seat_len // page] (the last row is the scratch seat padded rows point at,
    talker.py:29); default = identity pages. fuse_qk_norm_rope=False runs the layer norms, the q/k norms + RoPE and the
    MLP gate as separate PyTorch ops around the attention kernels, and fused_sampler=False samples with PyTorch ops and
    torch's generator instead of q3attn.sample_topk (same maths, another random stream; both kept to measure what the
    fusions save)."""

    def __init__(self, W, n_seats, seat_len=768, buckets=None, page=16, block_table=None, max_text=16,
                 temperature=0.9, top_k=50, rep_penalty=1.05, min_new=2, seed=0, fuse_qk_norm_rope=True,
                 fused_sampler=True):
        assert seat_len % page == 0
        self.W = W
        d, dt = W.device, W.dtype
        self.d, self.dt = d, dt
        self.n_seats, self.seat_len, self.page, self.P = n_seats, seat_len, page, seat_len // page
        self.H, self.nh, self.nkv, self.hd, self.ffn = W.H, W.heads, W.kv_heads, W.head_dim, W.ffn
        self.scale = float(self.hd) ** -0.5
        self.temperature, self.top_k, self.rep, self.min_new = temperature, top_k, rep_penalty, min_new
        S1 = n_seats + 1
        if block_table is None:
            block_table = (torch.arange(S1, dtype=torch.int32)[:, None] * self.P
                           + torch.arange(self.P, dtype=torch.int32)[None, :])
        self.seat_pages = block_table.to(device=d, dtype=torch.int32).contiguous()
        num_pages = int(self.seat_pages.max()) + 1
        self.kc = [torch.zeros(num_pages, page, self.nkv, self.hd, dtype=dt, device=d) for _ in W.layers]
        self.vc = [torch.zeros(num_pages, page, self.nkv, self.hd, dtype=dt, device=d) for _ in W.layers]
        self.pos = torch.zeros(S1, dtype=torch.int64, device=d)
        self.x_in = torch.zeros(S1, self.H, dtype=dt, device=d)
        self.seen = torch.zeros(S1, W.vocab, dtype=torch.bool, device=d)
        self.ngen = torch.zeros(S1, dtype=torch.int64, device=d)
        self.max_text = max_text
        self.trail = torch.zeros(S1, max_text + 1, self.H, dtype=dt, device=d)
        self.trail_len = torch.zeros(S1, dtype=torch.int64, device=d)
        sup = torch.zeros(W.vocab, device=d)
        sup[W.vocab - 1024:] = NEG
        sup[W.eos] = 0.0
        self.suppress = sup
        self.eos_col = torch.zeros(W.vocab, dtype=torch.bool, device=d)
        self.eos_col[W.eos] = True
        self.gen = torch.Generator(device=d)
        self.gen.manual_seed(seed)
        self.fused_sampler = fused_sampler
        self.rng = ops.SamplerRng(seed, d)       # the fused sampler's device random stream
        self.buckets = sorted(set(buckets or [1, 2, 4, 8, 16, 32, 64, 128, 256]))
        self.max_bs = self.buckets[-1]
        self.s_seat = torch.full((self.max_bs,), n_seats, dtype=torch.int64, device=d)
        self.o_codes = torch.zeros(self.max_bs, 16, dtype=torch.int64, device=d)
        self.fuse = fuse_qk_norm_rope
        self.cp = CodePredictor(W, self.max_bs, temperature=temperature, top_k=top_k,
                                fuse_qk_norm_rope=fuse_qk_norm_rope, fused_sampler=fused_sampler)
        self.graphs = {}
        self.pool = None

    # ------------------------------------------------------------------ talker maths
    def decode(self, x, cos, sin, pos, bt):
        """talker.py:63-80: x [B,H] -> post-norm hidden; appends each row's K/V at position pos and attends over pos+1."""
        B = x.shape[0]
        nq = self.nh * self.hd
        seqlens = pos.to(torch.int32)
        if self.fuse:
            # talker.py:66-80 with the q3attn row kernels (residual add + RMSNorm, SiLU gate) and the fused q/k norm +
            # RoPE + append + paged attention; x (a gathered copy) is the residual stream, updated in place
            r = None
            for l in range(len(self.W.layers)):
                w = self.W.layers[l]
                qkv = F.linear(ops.add_rms_norm(x, w.ln1, r), w.qkv)                      # talker.py:68
                o = ops.paged_decode_qkv(qkv, w.qn, w.kn, cos, sin, self.kc[l], self.vc[l], seqlens, bt,  # :69-77
                                         self.scale)
                h = ops.add_rms_norm(x, w.ln2, F.linear(o.reshape(B, nq), w.o))           # :78-79
                r = F.linear(ops.silu_mul(F.linear(h, w.gu)), w.down)
            return ops.add_rms_norm(x, self.W.norm, r)
        for l in range(len(self.W.layers)):   # the same maths as separate PyTorch ops
            w = self.W.layers[l]
            qkv = F.linear(rms(x, w.ln1), w.qkv)
            q, k, v = _split_qkv(qkv, w, cos, sin, B, self.nh, self.nkv, self.hd)
            o = ops.paged_decode_append(q, k, v, self.kc[l], self.vc[l], seqlens, bt, self.scale, 0)
            x = x + F.linear(o.reshape(B, nq), w.o)
            x = x + mlp(rms(x, w.ln2), w, self.ffn)
        return rms(x, self.W.norm)

    def _cb0_logits(self, h, seat):
        """talker.py:90-94."""
        lg = F.linear(h, self.W.codec_head).float()
        lg = torch.where(self.seen[seat], torch.where(lg < 0, lg * self.rep, lg / self.rep), lg) + self.suppress
        return lg.masked_fill((self.ngen[seat] < self.min_new)[:, None] & self.eos_col[None, :], NEG)

    def _tail(self, h, seat):
        """talker.py:96-105."""
        if self.fused_sampler:   # _cb0_logits' processing, the top-k draw and codec_emb[c0] in one launch
            c0, e0 = ops.sample_topk(F.linear(h, self.W.codec_head), self.temperature, self.top_k, self.rng,
                                     seen=self.seen, seat=seat, rep_penalty=self.rep, bias=self.suppress,
                                     ngen=self.ngen, min_new=self.min_new, eos=self.W.eos, emb=self.W.codec_emb)
        else:
            c0, e0 = sample_topk(self._cb0_logits(h, seat), self.temperature, self.top_k, self.gen), None
        g = self.ngen[seat]
        self.seen.index_put_((seat, c0), self.eos_col.new_ones(()).expand_as(c0))
        self.ngen.index_copy_(0, seat, g + 1)
        codes, acc = self.cp.run(h, c0, self.rng if self.fused_sampler else self.gen, e0)
        t = self.trail[seat, torch.minimum(g, self.trail_len[seat])]
        self.x_in.index_copy_(0, seat, acc + t)
        return torch.cat([c0[:, None], codes], 1)

    def _frame(self, B):
        """talker.py:107-112."""
        seat = self.s_seat[:B]
        pos = self.pos[seat]
        h = self.decode(self.x_in[seat], self.W.cos[pos][:, None, :], self.W.sin[pos][:, None, :], pos,
                        self.seat_pages[seat])
        self.pos.index_copy_(0, seat, torch.where(seat == self.n_seats, 0, pos + 1))   # scratch seat stays at 0
        self.o_codes[:B].copy_(self._tail(h, seat))

    # ------------------------------------------------------------------ graphs
    @torch.inference_mode()
    def capture(self, buckets=None):
        """talker.py:115-129: warm each bucket on the scratch seat only, then capture one graph per bucket."""
        cap = torch.cuda.Stream(device=self.d)
        for B in reversed(buckets or self.buckets):
            self.s_seat.fill_(self.n_seats)
            self.pos[self.n_seats] = 0
            with torch.cuda.stream(cap):
                for _ in range(2):
                    self._frame(B)
                    self.pos[self.n_seats] = 0
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            g.register_generator_state(self.gen)
            with torch.cuda.graph(g, pool=self.pool, stream=cap):
                self._frame(B)
            if self.pool is None:
                self.pool = g.pool()
            self.graphs[B] = g
        self.pos[self.n_seats] = 0
        self.ngen[self.n_seats] = 0
        self.seen[self.n_seats] = False
        torch.cuda.synchronize()

    @torch.inference_mode()
    def step(self, seats):
        """talker.py:132-138: one frame for the listed seats (graph replay); returns a view of the codes [B, 16]."""
        B = len(seats)
        bs = next(b for b in self.buckets if b >= B)
        self.pos[self.n_seats] = 0
        self.s_seat[:bs].fill_(self.n_seats)
        self.s_seat[:B].copy_(torch.as_tensor(seats, dtype=torch.int64), non_blocking=False)
        self.graphs[bs].replay()
        return self.o_codes[:B]

    # ------------------------------------------------------------------ state helpers
    @torch.inference_mode()
    def load_history(self, kv):
        """Fill every seat's K/V pages from kv [2, layers, n_seats + 1, seat_len, 8, 128] (through the block table)."""
        for l in range(len(self.W.layers)):
            for s in range(self.n_seats + 1):
                rows = self.seat_pages[s].long()
                self.kc[l][rows] = kv[0, l, s].view(self.P, self.page, self.nkv, self.hd).to(self.d, self.dt)
                self.vc[l][rows] = kv[1, l, s].view(self.P, self.page, self.nkv, self.hd).to(self.d, self.dt)

    @torch.inference_mode()
    def load_history_block(self, seed, ctx, seats=None, chunk=64):
        """Fill seats' K/V pages (positions 0..ctx[s]-1, through the block table) with synth.history_block rows,
        generated on the device in chunks of seats; ctx is a CPU tensor over all seats."""
        from q3attn import synth
        seats = list(range(self.n_seats)) if seats is None else list(seats)
        for l in range(len(self.W.layers)):
            for a in range(0, len(seats), chunk):
                sc = torch.tensor(seats[a:a + chunk], dtype=torch.int64)
                n = int(ctx[sc].max())
                if n == 0:
                    continue
                pos = torch.arange(n, device=self.d)
                valid = pos[None, :] < ctx[sc].to(self.d)[:, None]                          # [c, n]
                bt = self.seat_pages[sc.to(self.d)].long()                                  # [c, P]
                rows = bt.gather(1, (pos // self.page)[None, :].expand(len(sc), n)) * self.page + pos % self.page
                for kv, pool in ((0, self.kc[l]), (1, self.vc[l])):
                    vals = synth.history_block(seed, l, kv, sc, n, self.d)                  # [c, n, 8, 128]
                    pool.view(-1, self.nkv, self.hd)[rows[valid]] = vals[valid].to(self.dt)
