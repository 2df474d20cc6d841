"""Generate the golden fixtures by running the REFERENCE engine's own fp32 code on seeded inputs.

Run where the reference checkout is readable, with Q3_REFERENCE set to its directory:
    Q3_REFERENCE=<reference checkout> python tests/golden/make_golden.py
It imports engine.talker / engine.arrivals / engine.code_predictor from the reference (read-only; flash-attn and triton
only need to import) and calls:
  * Talker._attn_ref            (engine/talker.py:82-88)      paged decode on page-gathered caches  -> decode_c1.npz
  * FastAdmit._attn_ref         (engine/arrivals.py:125-131)  prefix / causal prefill              -> prefill.npz
  * CodePredictor._post         (engine/code_predictor.py:44-50) with identity o-proj and a zero MLP, so it returns
                                 the attention expression of code_predictor.py:46-47 exactly     -> cp_attn.npz
  * Talker._frame               (engine/talker.py:107-112) + CodePredictor.run, fp32, greedy (top_k=1), on random-init
                                 weights and a synthetic K/V history                              -> frame_*.npz
  * Talker._cb0_logits + sample_topk (engine/talker.py:90-94, engine/ops.py:68-76), greedy      -> sampler.npz
  * FastAdmit._run with the per-voice prefix from Talker.prefill_hidden (engine/arrivals.py:85-91, 133-152),
                                 fp32                                                             -> admit.npz
  * StreamDecoder._step / StreamCore.forward in ring mode on a small decoder (engine/decoder_stream.py:134-181),
                                 fp32                                                             -> ring.npz
Inputs are regenerated from seeds by q3attn.synth / q3attn.weights (torch CPU generators); each fixture stores a
checksum of its inputs so a generator mismatch is detected before outputs are compared. The GPU box never runs this.
"""
import hashlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "qwen3-tts-engine_b200"))
from q3attn import synth, weights  # noqa: E402

REF = os.environ.get("Q3_REFERENCE")   # the reference checkout (only the generators below need it)


def digest(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.detach().contiguous().float().numpy().tobytes())
    return h.hexdigest()[:32]


def b16(t: torch.Tensor) -> torch.Tensor:
    """fp32 values rounded to the nearest bf16: the inputs a bf16 kernel sees, so its output can be held to the bf16
    output tolerance against the reference's fp32 result on exactly those inputs."""
    return t.to(torch.bfloat16).float()


def ref_modules():
    if not REF:
        raise RuntimeError("set Q3_REFERENCE to the reference checkout to regenerate the fixtures")
    sys.path.insert(0, REF)
    from engine import talker, arrivals, code_predictor   # noqa: F401
    return talker, arrivals, code_predictor


# --------------------------------------------------------------------------- decode (C1)
def c1_inputs(seed=1):
    lay = synth.c1_layout(seed)
    d = synth.decode_case(seed, lay, scale=1.0, dtype=torch.float32)
    return lay, d


def gen_decode(talker):
    out = {}
    for seed in (1, 11, 12):
        lay, d = c1_inputs(seed)
        B, page = lay.B, lay.page
        # the reference reads a contiguous per-seat slice: lay each seat's gathered tokens out back to back
        rowsK, rowsV, slot, base = [], [], [], 0
        for b in range(B):
            n = int(lay.ctx[b])
            pg = lay.block_table[b, : (n + page - 1) // page].long()
            rowsK.append(d["k_pool"][pg].reshape(-1, 8, 128)[:n])
            rowsV.append(d["v_pool"][pg].reshape(-1, 8, 128)[:n])
            slot.append(base + n - 1)
            base += n
        ns = types.SimpleNamespace(kc=[torch.cat(rowsK)], vc=[torch.cat(rowsV)], nkv=8, hd=128, nh=16, scale=128 ** -0.5)
        o = talker.Talker._attn_ref(ns, d["q"], 0, torch.tensor(slot), lay.ctx)
        out[f"s{seed}_out"] = o.numpy()
        ns.kc, ns.vc = [b16(ns.kc[0])], [b16(ns.vc[0])]          # the same case on bf16-representable inputs
        out[f"s{seed}_b16_out"] = talker.Talker._attn_ref(ns, b16(d["q"]), 0, torch.tensor(slot), lay.ctx).numpy()
        out[f"s{seed}_ctx"] = lay.ctx.numpy()
        out[f"s{seed}_bt"] = lay.block_table.numpy()
        out[f"s{seed}_digest"] = np.array(digest(d["q"], d["k_pool"], d["v_pool"]))
    np.savez_compressed(os.path.join(HERE, "decode_c1.npz"), **out)


# --------------------------------------------------------------------------- prefill
PREFILL_CASES = {          # name: (seed, S, R, k)
    "arrivals": (21, 2, 42, 35),     # FastAdmit shape: R new positions over k cached prefix positions
    "causal": (22, 1, 77, 0),        # eager prompt prefill (no prefix)
    "ragged": (23, 3, 17, 5),
}


def prefill_inputs(seed, S, R, k):
    g = synth.cpu_gen(seed)
    q = synth.randn((S, R, 16, 128), g, 0.5)
    K = synth.randn((S, k + R, 8, 128), g, 0.5)
    V = synth.randn((S, k + R, 8, 128), g, 0.5)
    return q, K, V


def gen_prefill(arrivals):
    out = {}
    for name, (seed, S, R, k) in PREFILL_CASES.items():
        q, K, V = prefill_inputs(seed, S, R, k)
        ns = types.SimpleNamespace(T=types.SimpleNamespace(nkv=8, nh=16, hd=128, scale=128 ** -0.5))
        o = arrivals.FastAdmit._attn_ref(ns, q, K, V)
        out[f"{name}_out"] = o.numpy()
        out[f"{name}_b16_out"] = arrivals.FastAdmit._attn_ref(ns, b16(q), b16(K), b16(V)).numpy()
        out[f"{name}_digest"] = np.array(digest(q, K, V))
    np.savez_compressed(os.path.join(HERE, "prefill.npz"), **out)


# --------------------------------------------------------------------------- code predictor attention
def gen_cp(code_predictor):
    out = {}
    B = 8
    for p in range(16):
        d = synth.cp_case(40 + p, B, dtype=torch.float32)
        cp = object.__new__(code_predictor.CodePredictor)
        cp.nh, cp.nkv, cp.hd, cp.scale, cp.ffn = 16, 8, 128, 128 ** -0.5, 8
        mask = torch.full((16, 16), float("-inf")).triu(1)
        x = torch.zeros(B, 2048)
        args = (mask[p], torch.eye(2048), torch.ones(2048), torch.zeros(16, 2048), torch.zeros(2048, 8))
        o = code_predictor.CodePredictor._post(cp, x, d["q"], d["K"], d["V"], *args)
        out[f"p{p}_out"] = o.numpy()
        out[f"p{p}_b16_out"] = code_predictor.CodePredictor._post(cp, x, b16(d["q"]), b16(d["K"]), b16(d["V"]),
                                                                  *args).numpy()
        out[f"p{p}_digest"] = np.array(digest(d["q"], d["K"], d["V"]))
    np.savez_compressed(os.path.join(HERE, "cp_attn.npz"), **out)


# --------------------------------------------------------------------------- full frame (e2e)
FRAME_CASES = {
    # name: (size, talker layers (None = all), n_seats, live seats, bucket, seat_len, ctx range, frames, seed)
    "frame06": ("0.6B", None, 40, 29, 32, 512, (100, 400), 2, 7),
    "frame17": ("1.7B", 2, 12, 5, 8, 512, (50, 300), 2, 8),
}


def frame_state(size, n_layers, n_seats, n_live, seat_len, ctx_rng, seed):
    """Seeded synthetic engine state: bf16-rounded weights, K/V history per seat (N(0,1)*0.5), pending inputs,
    trailing text, generation counters. Returns plain fp32 tensors in the reference's identity layout."""
    W = weights.cast(weights.cast(weights.random_weights(seed, size, max_pos=seat_len + 64, n_layers=n_layers),
                                  torch.bfloat16), torch.float32)
    g = synth.cpu_gen(seed + 500)
    S1 = n_seats + 1
    nl = len(W.layers)
    live = torch.randperm(n_seats, generator=g)[:n_live]
    ctx = torch.zeros(S1, dtype=torch.int64)
    ctx[live] = torch.randint(ctx_rng[0], ctx_rng[1] + 1, (n_live,), generator=g)
    kv = synth.randn((2, nl, S1, seat_len, 8, 128), g, 0.5, torch.bfloat16).float()
    pos_idx = torch.arange(seat_len)[None, :]
    kv = kv * (pos_idx < ctx[:, None]).float()[None, None, :, :, None, None]      # positions >= ctx start empty
    x_in = synth.randn((S1, W.H), g, 0.1, torch.bfloat16).float()
    max_text = 16
    trail = synth.randn((S1, max_text + 1, W.H), g, 0.02, torch.bfloat16).float()
    trail_len = torch.randint(0, max_text + 1, (S1,), generator=g)
    ngen = torch.randint(0, 6, (S1,), generator=g)
    return W, dict(live=live, ctx=ctx, kv=kv, x_in=x_in, trail=trail, trail_len=trail_len, ngen=ngen, max_text=max_text)


def ref_talker(talker_mod, code_predictor_mod, W, n_seats, seat_len, bucket, st, kc=None, vc=None):
    """A reference Talker built without CUDA (object.__new__ + the attributes of engine/talker.py:24-54), fp32, top_k=1.
    The K/V pools come from st["kv"] unless kc / vc (lists of per-layer pools in the reference layout) are given."""
    T = object.__new__(talker_mod.Talker)
    T.W = W
    T.d, T.dt = torch.device("cpu"), torch.float32
    T.n_seats, T.seat_len, T.page, T.P = n_seats, seat_len, 256, seat_len // 256
    T.H, T.nh, T.nkv, T.hd, T.ffn = W.H, W.heads, W.kv_heads, W.head_dim, W.ffn
    T.scale = float(T.hd) ** -0.5
    T.temperature, T.top_k, T.rep, T.min_new = 0.9, 1, 1.05, 2
    S1 = n_seats + 1
    if kc is None:
        kc = [st["kv"][0, l].reshape(S1 * T.P, 256, 8, 128).clone() for l in range(len(W.layers))]
        vc = [st["kv"][1, l].reshape(S1 * T.P, 256, 8, 128).clone() for l in range(len(W.layers))]
    T.kc, T.vc = kc, vc
    T.pos = st["ctx"].clone()
    T.x_in = st["x_in"].clone()
    T.seen = torch.zeros(S1, W.vocab, dtype=torch.bool)
    T.ngen = st["ngen"].clone()
    T.max_text = st["max_text"]
    T.trail = st["trail"].clone()
    T.trail_len = st["trail_len"].clone()
    T.seat_pages = (torch.arange(S1, dtype=torch.int32)[:, None] * T.P + torch.arange(T.P, dtype=torch.int32)[None, :]).contiguous()
    sup = torch.zeros(W.vocab)
    sup[W.vocab - 1024:] = float("-inf")
    sup[W.eos] = 0.0
    T.suppress = sup
    T.eos_col = torch.zeros(W.vocab, dtype=torch.bool)
    T.eos_col[W.eos] = True
    T.one = torch.ones(1, dtype=torch.int64)
    T.gen = torch.Generator().manual_seed(0)
    T.buckets = [bucket]
    T.max_bs = bucket
    T.s_seat = torch.full((bucket,), n_seats, dtype=torch.int64)
    T.o_codes = torch.zeros(bucket, 16, dtype=torch.int64)
    T.cp = code_predictor_mod.CodePredictor(W, bucket, compile_mode="off", temperature=0.9, top_k=1)
    T.decode = T._decode
    return T


def gen_frames(talker, code_predictor):
    for name, (size, nl, n_seats, n_live, bucket, seat_len, rng, frames, seed) in FRAME_CASES.items():
        W, st = frame_state(size, nl, n_seats, n_live, seat_len, rng, seed)
        T = ref_talker(talker, code_predictor, W, n_seats, seat_len, bucket, st)
        live = st["live"]
        T.s_seat[:n_live] = live
        codes, hs = [], []
        dec = T._decode
        T.decode = lambda *args: hs.append(dec(*args)) or hs[-1]   # record the talker hidden of each frame
        with torch.inference_mode():
            for f in range(frames):
                T.pos[n_seats] = 0
                T._frame(bucket)
                codes.append(T.o_codes[:n_live].clone())
            # continuous values of frame 1 for the live rows: talker hidden, raw codebook-0 logits, and the 15 CP logits
            # teacher-forced on the frame's own codes (CodePredictor.tf_logits, engine/code_predictor.py:74-82)
            h1 = hs[0][:n_live].clone()
            lg1 = torch.nn.functional.linear(h1, W.codec_head).float()
            cp1 = T.cp.tf_logits(h1, codes[0])
        # the rows the first frame appended (placement pin): K of layer 0 at each live seat's first new position
        slot0 = live * seat_len + st["ctx"][live]
        krow0 = T.kc[0].view(-1, 8, 128)[slot0]
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), codes=torch.stack(codes).numpy(), live=live.numpy(),
                            x_in=T.x_in[live].numpy(), pos=T.pos.numpy(), ngen=T.ngen.numpy(), krow0=krow0.numpy(),
                            h1=h1.numpy(), c0_logits1=lg1.numpy().astype(np.float16),
                            cp_tf_logits1=cp1.numpy().astype(np.float16),
                            digest=np.array(digest(st["kv"][:, :, :, :8], st["x_in"], W.layers[0].qkv, W.cp_head[3])))
        print(f"[golden] {name}: codes {tuple(torch.stack(codes).shape)}", flush=True)


# --------------------------------------------------------------------------- the config-5 frame (e2e criterion)
# The GPU side runs a 576-seat bucket (all seats live, ctx U[200,1200], 28 layers, 16-token shuffled pages); the
# reference computes `checked` of those seats (seats are independent, so their results do not depend on the others).
# The K/V history comes from synth.history_rows (a hash of the position, identical on the CPU and the GPU), so it is
# regenerated on both sides instead of stored.
FRAME_C5 = dict(size="0.6B", n_seats=576, checked=128, seat_len=1280, ctx=(200, 1200), frames=2, seed=9, n_full=16)


def c5_state(c=FRAME_C5):
    """bf16-rounded weights (fp32 tensors) and the state of all n_seats + 1 seats: ctx, pending inputs, trailing text,
    generation counters, and the checked seats (sorted)."""
    W = weights.cast(weights.cast(weights.random_weights(c["seed"], c["size"], max_pos=c["seat_len"] + 64),
                                  torch.bfloat16), torch.float32)
    g = synth.cpu_gen(c["seed"] + 500)
    n, S1 = c["n_seats"], c["n_seats"] + 1
    ctx = torch.zeros(S1, dtype=torch.int64)
    ctx[:n] = torch.randint(c["ctx"][0], c["ctx"][1] + 1, (n,), generator=g)
    sel = torch.randperm(n, generator=g)[:c["checked"]].sort().values
    max_text = 16
    x_in = synth.randn((S1, W.H), g, 0.1, torch.bfloat16).float()
    trail = synth.randn((S1, max_text + 1, W.H), g, 0.02, torch.bfloat16).float()
    trail_len = torch.randint(0, max_text + 1, (S1,), generator=g)
    ngen = torch.randint(0, 6, (S1,), generator=g)
    return W, dict(ctx=ctx, sel=sel, x_in=x_in, trail=trail, trail_len=trail_len, ngen=ngen, max_text=max_text)


def c5_history_digest(c=FRAME_C5, st=None, device="cpu"):
    """Digest of a few history rows (first checked seat, layers 0 and 27, K and V): pins the generator across devices."""
    seat = int(st["sel"][0])
    n = int(st["ctx"][seat])
    return digest(*[synth.history_rows(c["seed"], l, kv, seat, n, device).cpu() for l in (0, 27) for kv in (0, 1)])


def gen_frame_c5(talker, code_predictor):
    c = FRAME_C5
    W, st = c5_state(c)
    sel, n, L = st["sel"], c["checked"], c["seat_len"]
    P = L // 256
    # the checked seats' pools in the reference layout (seat i of the reference = seat sel[i]); only the history rows
    # are written (torch.empty pages never touched stay unbacked), and the reference reads no other row
    kc = [torch.empty((n + 1) * P, 256, 8, 128) for _ in W.layers]
    vc = [torch.empty((n + 1) * P, 256, 8, 128) for _ in W.layers]
    for l in range(len(W.layers)):
        for i, s in enumerate(sel.tolist()):
            m = int(st["ctx"][s])
            kc[l].view(-1, 8, 128)[i * L:i * L + m] = synth.history_rows(c["seed"], l, 0, s, m)
            vc[l].view(-1, 8, 128)[i * L:i * L + m] = synth.history_rows(c["seed"], l, 1, s, m)
    rows = torch.cat([sel, torch.tensor([c["n_seats"]])])        # + the scratch seat
    sub = dict(ctx=st["ctx"][rows].clone(), x_in=st["x_in"][rows], trail=st["trail"][rows],
               trail_len=st["trail_len"][rows], ngen=st["ngen"][rows], max_text=st["max_text"])
    sub["ctx"][n] = 0
    T = ref_talker(talker, code_predictor, W, n, L, n, sub, kc=kc, vc=vc)
    T.s_seat[:n] = torch.arange(n)
    codes, hs = [], []
    dec = T._decode
    T.decode = lambda *args: hs.append(dec(*args)) or hs[-1]
    with torch.inference_mode():
        for f in range(c["frames"]):
            T.pos[n] = 0
            T._frame(n)
            codes.append(T.o_codes[:n].clone())
        h1 = hs[0][:n].clone()
        lg1 = torch.nn.functional.linear(h1, W.codec_head).float()
        cp1 = T.cp.tf_logits(h1, codes[0])                          # engine/code_predictor.py:74-82
    top2 = cp1.topk(2, -1).values
    np.savez_compressed(os.path.join(HERE, "frame_c5.npz"), sel=sel.numpy(), codes=torch.stack(codes).numpy().astype(np.int16),
                        h1=h1.numpy(), c0_logits1=lg1.numpy().astype(np.float16),
                        cp_tf_argmax=cp1.argmax(-1).numpy().astype(np.int16),
                        cp_tf_gap=(top2[..., 0] - top2[..., 1]).numpy().astype(np.float16),
                        cp_tf_logits_head=cp1[:c["n_full"]].numpy().astype(np.float16),
                        digest=np.array(digest(st["x_in"], W.layers[0].qkv, W.cp_head[3])),
                        history_digest=np.array(c5_history_digest(c, st)))
    print(f"[golden] frame_c5: {n} of {c['n_seats']} seats, codes {tuple(torch.stack(codes).shape)}", flush=True)


# --------------------------------------------------------------------------- admission (shared prefix + graphed prefill)
ADMIT = dict(size="0.6B", n_layers=3, n_seats=6, seat_len=512, seed=21, k=35, R=42, seats=[1, 4, 2],
             slots=[0, 1, 0], bucket=4, n_ids=64)


def admit_inputs():
    """Seeded admission inputs: weights/state as frame_state, two voices' prefix embeddings [2, k, H], a text table
    [n_ids, H], the admitted rows' prompt ids [S, R+1] and trailing-text ids [S, max_text+1] + lengths (bf16 values)."""
    c = ADMIT
    W, st = frame_state(c["size"], c["n_layers"], c["n_seats"], 2, c["seat_len"], (50, 100), c["seed"])
    g = synth.cpu_gen(c["seed"] + 900)
    prefix = synth.randn((2, c["k"], W.H), g, 0.5, torch.bfloat16).float()
    tab = synth.randn((c["n_ids"], W.H), g, 0.5, torch.bfloat16).float()
    S = len(c["seats"])
    rem = torch.randint(0, c["n_ids"], (S, c["R"] + 1), generator=g)
    trail_ids = torch.randint(0, c["n_ids"], (S, st["max_text"] + 1), generator=g)
    tlen = torch.randint(0, st["max_text"] + 1, (S,), generator=g)
    return W, st, prefix, tab, rem, trail_ids, tlen


def gen_admit(talker, arrivals, code_predictor):
    """FastAdmit._run (engine/arrivals.py:133-152) in fp32 on a reference Talker, with the per-voice prefix K/V computed
    by Talker.prefill_hidden in the scratch seat (what voice_slot does, arrivals.py:85-91)."""
    c = ADMIT
    W, st, prefix, tab, rem, trail_ids, tlen = admit_inputs()
    T = ref_talker(talker, code_predictor, W, c["n_seats"], c["seat_len"], c["bucket"], st)
    k, R, nl, sl = c["k"], c["R"], len(W.layers), c["seat_len"]
    A = object.__new__(arrivals.FastAdmit)
    A.T, A.W, A.d, A.dt, A.k, A.R, A.L = T, W, torch.device("cpu"), torch.float32, k, R, k + R + 1
    A.pK = torch.zeros(nl, 2, k, 8, 128)
    A.pV = torch.zeros_like(A.pK)
    s = T.n_seats
    with torch.inference_mode():
        for slot in (0, 1):
            T.prefill_hidden([s], [prefix[slot]])
            for l in range(nl):
                A.pK[l, slot] = T.kc[l].view(-1, 8, 128)[s * sl:s * sl + k]
                A.pV[l, slot] = T.vc[l].view(-1, 8, 128)[s * sl:s * sl + k]
        S, B = c["bucket"], len(c["seats"])
        A.tab = tab
        A.crem = torch.zeros(2, R + 1, W.H)
        A.s_seat = torch.full((S,), c["n_seats"], dtype=torch.int64)
        A.s_seat[:B] = torch.tensor(c["seats"])
        A.s_slot = torch.zeros(S, dtype=torch.int64)
        A.s_slot[:B] = torch.tensor(c["slots"])
        A.s_rem = torch.zeros(S, R + 1, dtype=torch.int64)
        A.s_rem[:B] = rem
        A.s_trail = torch.zeros(S, st["max_text"] + 1, dtype=torch.int64)
        A.s_trail[:B] = trail_ids
        A.s_tlen = torch.zeros(S, dtype=torch.int64)
        A.s_tlen[:B] = tlen
        A.z_seen = torch.zeros(S, W.vocab, dtype=torch.bool)
        A.z_i = torch.zeros(S, dtype=torch.int64)
        A.c_pos = torch.full((S,), k + R, dtype=torch.int64)
        A.ar = torch.arange(k + R)[None, :]
        A.cos, A.sin = W.cos[k:k + R][None, :, None, :], W.sin[k:k + R][None, :, None, :]
        A.layer, A.post = A._layer, A._post
        T.seen[torch.tensor(c["seats"])] = True                                 # the reset must clear these
        A._run(S)
    seats = torch.tensor(c["seats"])
    out = {}
    for l in (0, nl - 1):                # the first layer and the deepest (fp16 keeps the fixture small)
        rows = (seats[:, None] * sl + torch.arange(k + R)[None, :]).reshape(-1)
        out[f"K{l}"] = T.kc[l].view(-1, 8, 128)[rows].view(B, k + R, 8, 128).numpy().astype(np.float16)
        out[f"V{l}"] = T.vc[l].view(-1, 8, 128)[rows].view(B, k + R, 8, 128).numpy().astype(np.float16)
    out.update(x_in=T.x_in[seats].numpy(), pos=T.pos.numpy(), trail=T.trail[seats].numpy(),
               trail_len=T.trail_len[seats].numpy(), ngen=T.ngen[seats].numpy(), seen=T.seen[seats].numpy(),
               digest=np.array(digest(prefix, tab, rem.float(), W.layers[0].qkv)))
    np.savez_compressed(os.path.join(HERE, "admit.npz"), **out)


# --------------------------------------------------------------------------- codec decoder: windowed ring attention
RING_CASE = dict(seed=31, S=3, D=256, H=4, hd=64, L=3, D0=32, C1=16, C2=8,
                 calls=[([0, 2, 1], 4)] * 23 + [([0, 2, 1], 1), ([2, 0], 2), ([0, 2, 1], 3)])


def ring_h(call: int, B: int, n: int, D: int, seed: int):
    """Seeded transformer input [B, n, D] of call `call` (regenerated identically by the GPU test)."""
    return synth.randn((B, n, D), synth.cpu_gen(seed * 1000 + call), 1.0)


def ring_model(seed, D, H, hd, L):
    """Decoder transformer layers with the attribute layout of the upstream modules StreamCore uses."""
    g = synth.cpu_gen(seed)
    N = types.SimpleNamespace

    def lin(i, o, std):
        m = torch.nn.Linear(i, o, bias=False)
        m.weight.data = torch.randn(o, i, generator=g) * std
        return m

    def norm():
        return N(weight=1 + 0.1 * torch.randn(D, generator=g), variance_epsilon=1e-5)
    layers = []
    for _ in range(L):
        layers.append(N(input_layernorm=norm(), post_attention_layernorm=norm(),
                        self_attn=N(q_proj=lin(D, H * hd, 0.06), k_proj=lin(D, H * hd, 0.06),
                                    v_proj=lin(D, H * hd, 0.06), o_proj=lin(H * hd, D, 0.06)),
                        self_attn_layer_scale=N(scale=0.5 + 0.1 * torch.randn(D, generator=g)),
                        mlp=N(gate_proj=lin(D, 2 * D, 0.06), up_proj=lin(D, 2 * D, 0.06), down_proj=lin(2 * D, D, 0.06)),
                        mlp_layer_scale=N(scale=0.5 + 0.1 * torch.randn(D, generator=g))))
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))
    return layers, inv_freq


def gen_ring(decoder_stream):
    """StreamDecoder._step + StreamCore.forward in ring mode (engine/decoder_stream.py:134-181, 325-339), fp32, on a
    small decoder: the transformer layers of ring_model, and around them the smallest stack forward() accepts (no
    upsampling, one conv, one SnakeBeta, the final conv). The transformer input of each call is replaced by seeded
    values (ring_h) and the transformer output is recorded at the input of output_proj."""
    c = RING_CASE
    D, H, hd, L, S = c["D"], c["H"], c["hd"], c["L"], c["S"]
    layers, inv_freq = ring_model(c["seed"], D, H, hd, L)
    core = object.__new__(decoder_stream.StreamCore)
    torch.nn.Module.__init__(core)
    core.dtype, core.nhwc, core.ring, core.lazy = torch.float32, False, True, False
    core.H, core.hd, core.L = H, hd, L
    core.layers = layers
    core.inv_freq = inv_freq
    core.rvq = torch.zeros(16, 4, c["D0"])
    core.rvq_off = (torch.arange(16) * 4)[None, :, None]
    core.pre_conv = torch.nn.Conv1d(c["D0"], c["D0"], 3)
    calls = {"i": 0}
    outs = []

    class SeededH(torch.nn.Module):
        def forward(self, x):
            h = ring_h(calls["i"], x.shape[0], x.shape[1], D, c["seed"])
            calls["i"] += 1
            return h

    class Record(torch.nn.Module):
        def forward(self, x):
            outs.append(x.clone())
            return torch.zeros(x.shape[0], x.shape[1], c["C1"])
    core.tr = types.SimpleNamespace(input_proj=SeededH(), norm=types.SimpleNamespace(weight=torch.ones(D),
                                                                                   variance_epsilon=1e-5),
                                    output_proj=Record())
    core.ups, core.blocks, core.rates = [], [], []
    core.conv0 = torch.nn.Conv1d(c["C1"], c["C2"], 7)
    core.fin_conv = torch.nn.Conv1d(c["C2"], 1, 7)
    core.sa0, core.sb0 = torch.ones(c["C2"], 1), torch.zeros(c["C2"], 1)
    dec = object.__new__(decoder_stream.StreamDecoder)
    dec.device, dec.dtype, dec.n_slots, dec.dummy = "cpu", torch.float32, S, S
    dec.core = dec.fn = core
    dec.pos = torch.zeros(S + 1, dtype=torch.long)
    R = decoder_stream.RING
    dec.state = [torch.zeros(S + 1, c["D0"], 2), torch.zeros(S + 1, R, L, H, hd), torch.zeros(S + 1, R, L, H, hd),
                 torch.zeros(S + 1, c["C1"], 6), torch.zeros(S + 1, c["C2"], 6)]
    with torch.inference_mode():
        for seats, n in c["calls"]:
            dec._step(torch.tensor(seats), torch.zeros(len(seats), 16, n, dtype=torch.long))
    assert calls["i"] == len(c["calls"])
    out = {f"h{k}": o.numpy().astype(np.float16) for k, o in enumerate(outs)}
    out["K_last"] = dec.state[1][:S, :, L - 1].numpy().astype(np.float16)      # the deepest layer's rings
    out["V_last"] = dec.state[2][:S, :, L - 1].numpy().astype(np.float16)
    out["pos"] = dec.pos.numpy()
    out["digest"] = np.array(digest(layers[0].self_attn.q_proj.weight, ring_h(0, 3, 4, D, c["seed"])))
    np.savez_compressed(os.path.join(HERE, "ring.npz"), **out)


# --------------------------------------------------------------------------- codebook-0 logit processing + greedy sampling
def gen_sampler(talker, ops_mod):
    """Talker._cb0_logits (engine/talker.py:90-94) with an identity codec_head, so its input row IS the logit row, and
    sample_topk (engine/ops.py:68-76) with top_k = 1 (greedy), on synth.sampler_case inputs."""
    out = {}
    for seed in (1, 2):
        d = synth.sampler_case(seed)
        V = d["logits"].shape[1]
        eos_col = torch.zeros(V, dtype=torch.bool)
        eos_col[d["eos"]] = True
        ns = types.SimpleNamespace(W=types.SimpleNamespace(codec_head=torch.eye(V)), seen=d["seen"], rep=d["rep"],
                                   suppress=d["suppress"], ngen=d["ngen"], min_new=d["min_new"], eos_col=eos_col)
        lg = talker.Talker._cb0_logits(ns, d["logits"], d["seat"])
        ids = ops_mod.sample_topk(lg, 0.9, 1, torch.Generator().manual_seed(0))
        out[f"s{seed}_processed"] = lg.numpy()
        out[f"s{seed}_greedy"] = ids.numpy()
        out[f"s{seed}_digest"] = np.array(digest(d["logits"], d["seen"], d["seat"], d["ngen"]))
    np.savez_compressed(os.path.join(HERE, "sampler.npz"), **out)


if __name__ == "__main__":
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    talker, arrivals, code_predictor = ref_modules()
    only = sys.argv[1:]
    if not only or "decode" in only:
        gen_decode(talker)
    if not only or "prefill" in only:
        gen_prefill(arrivals)
    if not only or "cp" in only:
        gen_cp(code_predictor)
    if not only or "frames" in only:
        gen_frames(talker, code_predictor)
    if not only or "frame_c5" in only:
        gen_frame_c5(talker, code_predictor)
    if not only or "admit" in only:
        gen_admit(talker, arrivals, code_predictor)
    if not only or "ring" in only:
        from engine import decoder_stream
        gen_ring(decoder_stream)
    if not only or "sampler" in only:
        from engine import ops as ref_ops
        gen_sampler(talker, ref_ops)
    print("[golden] done", flush=True)
