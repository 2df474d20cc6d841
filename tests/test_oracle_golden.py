"""CPU: the oracle restatement against fixtures produced by the reference's own code (tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest
import torch

import make_golden as mg
from oracle import attention as OA
from oracle.frame import FrameOracle
from q3attn import synth


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


@pytest.mark.parametrize("seed", [1, 11, 12])
def test_decode_c1_matches_reference(golden_dir, seed):
    g = _load(golden_dir, "decode_c1.npz")
    lay, d = mg.c1_inputs(seed)
    assert str(g[f"s{seed}_digest"]) == mg.digest(d["q"], d["k_pool"], d["v_pool"]), "input generator drifted"
    assert np.array_equal(g[f"s{seed}_ctx"], lay.ctx.numpy())
    assert np.array_equal(g[f"s{seed}_bt"], lay.block_table.numpy())
    o = OA.decode_attention(d["q"], d["k_pool"], d["v_pool"], lay.ctx, lay.block_table, 128 ** -0.5)
    np.testing.assert_allclose(o.numpy(), g[f"s{seed}_out"], rtol=1e-5, atol=1e-6)
    o = OA.decode_attention(mg.b16(d["q"]), mg.b16(d["k_pool"]), mg.b16(d["v_pool"]), lay.ctx, lay.block_table,
                            128 ** -0.5)
    np.testing.assert_allclose(o.numpy(), g[f"s{seed}_b16_out"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", list(mg.PREFILL_CASES))
def test_prefill_matches_reference(golden_dir, name):
    g = _load(golden_dir, "prefill.npz")
    q, K, V = mg.prefill_inputs(*mg.PREFILL_CASES[name])
    assert str(g[f"{name}_digest"]) == mg.digest(q, K, V)
    o = OA.prefill_prefix(q, K, V, 128 ** -0.5)
    np.testing.assert_allclose(o.numpy(), g[f"{name}_out"], rtol=1e-5, atol=1e-6)
    o = OA.prefill_prefix(mg.b16(q), mg.b16(K), mg.b16(V), 128 ** -0.5)
    np.testing.assert_allclose(o.numpy(), g[f"{name}_b16_out"], rtol=1e-5, atol=1e-6)


def test_prefill_varlen_equals_per_sequence(golden_dir):
    """The packed varlen form (talker.py:169) equals the per-sequence prefix form the reference fixture pins."""
    g = _load(golden_dir, "prefill.npz")
    seed, S, R, k = mg.PREFILL_CASES["ragged"]
    q, K, V = mg.prefill_inputs(seed, S, R, k)
    cu = torch.arange(S + 1, dtype=torch.int32) * R
    cp = torch.arange(S + 1, dtype=torch.int32) * k
    o = OA.prefill_varlen(q.reshape(S * R, 16, 128), K[:, k:].reshape(-1, 8, 128), V[:, k:].reshape(-1, 8, 128), cu,
                          128 ** -0.5, K[:, :k].reshape(-1, 8, 128), V[:, :k].reshape(-1, 8, 128), cp)
    np.testing.assert_allclose(o.numpy().reshape(S, R, 16, 128), g["ragged_out"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("p", range(16))
def test_cp_attention_matches_reference(golden_dir, p):
    g = _load(golden_dir, "cp_attn.npz")
    d = synth.cp_case(40 + p, 8, dtype=torch.float32)
    assert str(g[f"p{p}_digest"]) == mg.digest(d["q"], d["K"], d["V"])
    o = OA.cp_attention(d["q"], d["K"], d["V"], p + 1, 128 ** -0.5)
    np.testing.assert_allclose(o.numpy(), g[f"p{p}_out"], rtol=1e-5, atol=1e-6)
    o = OA.cp_attention(mg.b16(d["q"]), mg.b16(d["K"]), mg.b16(d["V"]), p + 1, 128 ** -0.5)
    np.testing.assert_allclose(o.numpy(), g[f"p{p}_b16_out"], rtol=1e-5, atol=1e-6)


def test_append_placement_identity_table_equals_flat_slot():
    """Through the identity table with 256-token pages the paged placement is the reference's flat slot
    seat*seat_len + pos (engine/talker.py:42, 109)."""
    S1, seat_len = 5, 512
    P = seat_len // 256
    bt = (torch.arange(S1, dtype=torch.int32)[:, None] * P + torch.arange(P, dtype=torch.int32)[None, :])
    for s in range(S1):
        for pos in (0, 1, 255, 256, 511):
            assert OA.slot_of(bt, s, pos, 256) == s * seat_len + pos


def _shuffled_table(n_rows, pages_per_seat, seed):
    g = synth.cpu_gen(seed)
    perm = torch.randperm(n_rows * pages_per_seat, generator=g)
    return perm.view(n_rows, pages_per_seat).to(torch.int32)


def run_frame_oracle(name, page=16):
    """The oracle's frame step over a SHUFFLED paged layout, fed the same synthetic state as the reference fixture."""
    size, nl, n_seats, n_live, bucket, seat_len, rng, frames, seed = mg.FRAME_CASES[name]
    W, st = mg.frame_state(size, nl, n_seats, n_live, seat_len, rng, seed)
    S1 = n_seats + 1
    pps = seat_len // page
    bt = _shuffled_table(S1, pps, seed + 77)
    O = FrameOracle(W, n_seats, bt, page, S1 * pps, bucket, max_text=st["max_text"])
    for l in range(len(W.layers)):
        for s in range(S1):
            rows = bt[s].long()
            O.kc[l][rows] = st["kv"][0, l, s].view(pps, page, 8, 128)
            O.vc[l][rows] = st["kv"][1, l, s].view(pps, page, 8, 128)
    O.pos[:] = st["ctx"]
    O.x_in[:] = st["x_in"]
    O.ngen[:] = st["ngen"]
    O.trail[:] = st["trail"]
    O.trail_len[:] = st["trail_len"]
    live = st["live"]
    seat = torch.full((bucket,), n_seats, dtype=torch.int64)
    seat[:n_live] = live
    codes = []
    for _ in range(frames):
        O.pos[n_seats] = 0
        codes.append(O.frame(seat)[:n_live])
    return W, st, O, torch.stack(codes), bt


@pytest.mark.parametrize("name", ["frame17", "frame06"])
def test_frame_oracle_matches_reference(golden_dir, name):
    g = _load(golden_dir, f"{name}.npz")
    W, st, O, codes, bt = run_frame_oracle(name)
    assert str(g["digest"]) == mg.digest(st["kv"][:, :, :, :8], st["x_in"], W.layers[0].qkv, W.cp_head[3])
    assert np.array_equal(codes.numpy(), g["codes"]), "greedy codes differ from the reference frame"
    live = st["live"]
    np.testing.assert_allclose(O.x_in[live].numpy(), g["x_in"], rtol=1e-4, atol=1e-5)
    n_seats = mg.FRAME_CASES[name][2]
    assert np.array_equal(O.pos[:n_seats].numpy(), g["pos"][:n_seats])
    assert np.array_equal(O.ngen[:n_seats].numpy(), g["ngen"][:n_seats])
    # placement pin: the rows the first frame appended sit where the reference put them, through the shuffled table
    page = 16
    kr = torch.stack([O.kc[0].view(-1, 8, 128)[OA.slot_of(bt, int(s), int(st["ctx"][s]), page)] for s in live])
    np.testing.assert_allclose(kr.numpy(), g["krow0"], rtol=1e-5, atol=1e-6)


def test_c5_frame_fixture_inputs_regenerate(golden_dir):
    """The config-5 frame fixture's inputs come back from their seeds: the engine state and the hashed K/V history
    (the GPU test regenerates the same history on the device and checks the same digest there)."""
    g = _load(golden_dir, "frame_c5.npz")
    W, st = mg.c5_state(mg.FRAME_C5)
    assert str(g["digest"]) == mg.digest(st["x_in"], W.layers[0].qkv, W.cp_head[3])
    assert str(g["history_digest"]) == mg.c5_history_digest(mg.FRAME_C5, st)
    assert np.array_equal(g["sel"], st["sel"].numpy())
