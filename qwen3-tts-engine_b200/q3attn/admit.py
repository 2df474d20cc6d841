"""Admission on the q3attn kernels: the shared-prefix K/V cache and graphed prefill of engine/arrivals.py (FastAdmit).

Mirrors FastAdmit (engine/arrivals.py:43-167). The K/V of the k prompt positions that every request of one
(voice, language) shares are computed once per slot (register_prefix: the prefix prefilled into the scratch seat, as
voice_slot does with T.prefill_hidden, arrivals.py:85-91) and kept as pK/pV [layers, slots, k, 8, 128]. Admitting S
seats is one CUDA graph per S bucket (arrivals.py:154-167) whose body (_run, arrivals.py:133-152):
  1. resets each seat's sampling state and trailing text (arrivals.py:136-137);
  2. copies the slot's prefix K/V of every layer into the seats' pages in ONE launch (q3attn.kv_copy_prefix);
  3. runs the R remaining prompt positions through the layers: per layer the residual add + RMSNorm (one launch), the
     QKV GEMM, the q/k norm + RoPE in place (one launch), then ONE paged prefill launch that attends over prefix (in the pages) + new rows with bottom-right causal alignment and
     writes the new K/V rows (arrivals.py:139-148); the last layer only writes its K/V rows (arrivals.py:146);
  4. sets pos = k + R and the pending talker input to the last prompt position (arrivals.py:149-151).
The prompt embeddings (text table + codec track, arrivals.py:137-139) and trailing-text rows are inputs: building them
is the prompt builder's job, not the attention path's.
"""
import torch
import torch.nn.functional as F

from . import ops


class Admit:
    def __init__(self, talker, k: int, R: int, max_slots: int = 8, buckets=(1, 2, 4, 8)):
        T = talker
        W = T.W
        d, dt = T.d, T.dt
        self.T, self.W, self.k, self.R = T, W, int(k), int(R)
        self.nl = len(W.layers)
        self.buckets = sorted(buckets)
        S = self.buckets[-1]
        self.pK = torch.zeros(self.nl, max_slots, k, T.nkv, T.hd, dtype=dt, device=d)
        self.pV = torch.zeros_like(self.pK)
        self.k_ptrs = ops.pool_pointers(T.kc)
        self.v_ptrs = ops.pool_pointers(T.vc)
        self.pool_shape = tuple(T.kc[0].shape)
        # static inputs of the graphs (arrivals.py:100-106)
        self.s_seat = torch.full((S,), T.n_seats, dtype=torch.int64, device=d)
        self.s_slot = torch.zeros(S, dtype=torch.int64, device=d)
        self.s_x = torch.zeros(S, R + 1, T.H, dtype=dt, device=d)            # prompt embeddings of positions k..k+R
        self.s_trail = torch.zeros(S, T.max_text + 1, T.H, dtype=dt, device=d)
        self.s_tlen = torch.zeros(S, dtype=torch.int64, device=d)
        self.z_seen = torch.zeros(S, W.vocab, dtype=torch.bool, device=d)
        self.z_i = torch.zeros(S, dtype=torch.int64, device=d)
        self.c_pos = torch.full((S,), k + R, dtype=torch.int64, device=d)
        # per-token rotary rows of positions k..k+R-1, and the row bookkeeping of a bucket of S sequences
        self.cos_new, self.sin_new = W.cos[k:k + R], W.sin[k:k + R]
        self.meta = {}
        for b in self.buckets + [1]:
            self.meta[("new", b)] = self._meta(b, R, k)
        self.graphs, self.pool = {}, None

    def _meta(self, S, n, prefix):
        d = self.T.d
        return dict(cu=torch.arange(S + 1, dtype=torch.int32, device=d) * n,
                    plen=torch.full((S,), prefix, dtype=torch.int32, device=d),
                    pos=(torch.arange(n, dtype=torch.int32, device=d) + prefix).repeat(S),
                    row_of=torch.arange(S, dtype=torch.int32, device=d).repeat_interleave(n))

    # ------------------------------------------------------------------ maths
    def _layers(self, x, seats, n, prefix, meta, cos, sin):
        """x [S, n, H] at positions prefix..prefix+n-1 of `seats` (int64 [S]); writes every layer's K/V rows of those
        positions; attends (all but the last layer) over the seats' first prefix positions (already in the pages) and
        the new rows. arrivals.py:112-123 (_layer, _post) + 139-148."""
        T = self.T
        S = x.shape[0]
        nq, nk = T.nh * T.hd, T.nkv * T.hd
        seat32 = seats.to(torch.int32)
        seat_rows = seat32[meta["row_of"]]
        bt = T.seat_pages
        c = cos.repeat(S, 1)
        s = sin.repeat(S, 1)
        xf = x.reshape(S * n, T.H).clone()                      # the residual stream, updated in place
        r = None
        for l in range(self.nl):
            w = self.W.layers[l]
            qkv = F.linear(ops.add_rms_norm(xf, w.ln1, r), w.qkv)
            ops.qk_norm_rope_(qkv, w.qn, w.kn, c, s)            # arrivals.py:114-115, in place on the q and k heads
            q = qkv[:, :nq].view(-1, T.nh, T.hd)
            kk = qkv[:, nq:nq + nk].view(-1, T.nkv, T.hd)
            v = qkv[:, nq + nk:].view(-1, T.nkv, T.hd)
            if l == self.nl - 1:                 # arrivals.py:146: only the K/V of the last layer are needed
                ops.kv_append_paged(kk, v, T.kc[l], T.vc[l], meta["pos"], bt, seat_rows)
                break
            o = ops.prefill_paged(q, kk, v, T.kc[l], T.vc[l], meta["cu"], meta["cu"], n, meta["plen"], seat32, bt,
                                  T.scale, True, True)
            h = ops.add_rms_norm(xf, w.ln2, F.linear(o.reshape(S * n, nq), w.o))
            r = F.linear(ops.silu_mul(F.linear(h, w.gu)), w.down)

    @torch.inference_mode()
    def register_prefix(self, slot: int, prefix: torch.Tensor):
        """Compute and keep the prefix K/V of one (voice, language) (arrivals.py:67-96): prefix [k, H] embeddings."""
        T = self.T
        k = self.k
        assert prefix.shape == (k, T.H)
        s = torch.tensor([T.n_seats], dtype=torch.int64, device=T.d)        # the scratch seat, as voice_slot uses
        meta = self._meta(1, k, 0)
        self._layers(prefix.to(T.dt)[None], s, k, 0, meta, self.W.cos[:k], self.W.sin[:k])
        pos = torch.arange(k, device=T.d)
        rows = T.seat_pages[T.n_seats].long()[pos // T.page] * T.page + pos % T.page
        for l in range(self.nl):
            self.pK[l, slot] = T.kc[l].view(-1, T.nkv, T.hd)[rows]
            self.pV[l, slot] = T.vc[l].view(-1, T.nkv, T.hd)[rows]
        T.pos[T.n_seats] = 0

    def _run(self, S):
        """arrivals.py:133-152 for the first S rows of the static inputs."""
        T = self.T
        seat, slot = self.s_seat[:S], self.s_slot[:S]
        R = self.R
        T.seen.index_copy_(0, seat, self.z_seen[:S])
        T.ngen.index_copy_(0, seat, self.z_i[:S])
        T.trail.index_copy_(0, seat, self.s_trail[:S])
        T.trail_len.index_copy_(0, seat, self.s_tlen[:S])
        ops.kv_copy_prefix(self.pK, self.pV, self.k_ptrs, self.v_ptrs, self.pool_shape, seat, slot, T.seat_pages)
        self._layers(self.s_x[:S, :R], seat, R, self.k, self.meta[("new", S)], self.cos_new, self.sin_new)
        T.pos.index_copy_(0, seat, self.c_pos[:S])
        T.x_in.index_copy_(0, seat, self.s_x[:S, R])
        T.pos[T.n_seats:].zero_()

    # ------------------------------------------------------------------ graphs
    @torch.inference_mode()
    def capture(self):
        """arrivals.py:154-167: warm each bucket on the scratch seat, then one graph per bucket."""
        T = self.T
        cap = torch.cuda.Stream(device=T.d)
        for S in reversed(self.buckets):
            self.s_seat.fill_(T.n_seats)
            with torch.cuda.stream(cap):
                for _ in range(2):
                    self._run(S)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=self.pool, stream=cap):
                self._run(S)
            if self.pool is None:
                self.pool = g.pool()
            self.graphs[S] = g
        torch.cuda.synchronize()

    @torch.inference_mode()
    def admit(self, seats, slots, x, trail, trail_len):
        """Admit len(seats) sequences: x [n, R+1, H] prompt embeddings of positions k..k+R, trail [n, max_text+1, H],
        trail_len [n]. Replays the smallest bucket graph that fits (padded rows use the scratch seat)."""
        n = len(seats)
        S = next(b for b in self.buckets if b >= n)
        self.s_seat.fill_(self.T.n_seats)
        self.s_seat[:n].copy_(torch.as_tensor(seats, dtype=torch.int64))
        self.s_slot.zero_()
        self.s_slot[:n].copy_(torch.as_tensor(slots, dtype=torch.int64))
        self.s_x[:n].copy_(x)
        self.s_trail[:n].copy_(trail)
        self.s_tlen[:n].copy_(torch.as_tensor(trail_len, dtype=torch.int64))
        self.graphs[S].replay() if S in self.graphs else self._run(S)
