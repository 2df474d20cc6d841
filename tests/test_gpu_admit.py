"""GPU parity: admission on the q3attn kernels (engine/arrivals.py FastAdmit): the one-launch shared-prefix copy
(bit-exact placement through the block table) and the whole graphed admission against what the reference's own
FastAdmit._run computed in fp32, with the per-voice prefix from Talker.prefill_hidden (tests/golden/admit.npz)."""
import os

import numpy as np
import pytest
import torch

import make_golden as mg
from helpers import bits_equal
from oracle import attention as OA
from q3attn import synth, weights

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def q3():
    import q3attn
    q3attn._lib.load()
    return q3attn


@pytest.mark.parametrize("page", [16, 1, 256])
def test_prefix_copy_places_every_layer_row(q3, page):
    L, slots, k, B = 5, 3, 37, 4
    pps = (512 + page - 1) // page
    g = synth.cpu_gen(70 + page)
    n_pages = (B + 2) * pps
    bt = torch.randperm(n_pages, generator=g)[: (B + 2) * pps].view(B + 2, pps).to(torch.int32)
    pools_k = [synth.randn((n_pages, page, 8, 128), g, 1.0, torch.bfloat16) for _ in range(L)]
    pools_v = [synth.randn((n_pages, page, 8, 128), g, 1.0, torch.bfloat16) for _ in range(L)]
    src_k = synth.randn((L, slots, k, 8, 128), g, 1.0, torch.bfloat16)
    src_v = synth.randn((L, slots, k, 8, 128), g, 1.0, torch.bfloat16)
    seat = torch.tensor([3, 0, 5, 1], dtype=torch.int64)
    slot = torch.tensor([2, 0, 2, 1], dtype=torch.int64)
    gk = [p.to(DEV) for p in pools_k]
    gv = [p.to(DEV) for p in pools_v]
    q3.ops.kv_copy_prefix(src_k.to(DEV), src_v.to(DEV), q3.ops.pool_pointers(gk), q3.ops.pool_pointers(gv),
                          gk[0].shape, seat.to(DEV), slot.to(DEV), bt.to(DEV))
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0
    pos = torch.arange(k, dtype=torch.int32)
    for l in range(L):
        rk, rv = pools_k[l].clone(), pools_v[l].clone()
        for b in range(B):
            OA.append_paged(rk, rv, src_k[l, slot[b]], src_v[l, slot[b]], pos, bt[[int(seat[b])] * k])
        assert bits_equal(gk[l], rk) and bits_equal(gv[l], rv), f"layer {l}"


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm())


def test_admission_matches_reference_fastadmit(q3, golden_dir):
    from q3attn.admit import Admit
    from frame_harness import Talker
    c = mg.ADMIT
    W, st, prefix, tab, rem, trail_ids, tlen = mg.admit_inputs()
    gold = np.load(os.path.join(golden_dir, "admit.npz"))
    assert str(gold["digest"]) == mg.digest(prefix, tab, rem.float(), W.layers[0].qkv), "input generator drifted"
    Wg = weights.cast(W, torch.bfloat16, DEV)
    n_seats, sl, k, R = c["n_seats"], c["seat_len"], c["k"], c["R"]
    page = 16
    table = torch.randperm((n_seats + 1) * (sl // page), generator=synth.cpu_gen(5)).view(n_seats + 1, sl // page)
    T = Talker(Wg, n_seats, seat_len=sl, buckets=[4], page=page, block_table=table.to(torch.int32), top_k=1)
    T.load_history(st["kv"])
    T.pos.copy_(st["ctx"].to(DEV))
    T.seen[torch.tensor(c["seats"])] = True
    A = Admit(T, k, R, max_slots=2, buckets=[c["bucket"]])
    for slot in (0, 1):
        A.register_prefix(slot, prefix[slot].to(DEV, torch.bfloat16))
    A.capture()
    x = tab[rem].to(DEV, torch.bfloat16)
    A.admit(c["seats"], c["slots"], x, tab[trail_ids].to(DEV, torch.bfloat16), tlen)
    torch.cuda.synchronize()
    assert q3._lib.read_status() == 0

    seats = torch.tensor(c["seats"])
    nl = len(W.layers)
    for l, tol in ((0, 1.5e-2), (nl - 1, 4e-2)):
        pos = torch.arange(k + R)
        rows = (table[seats][:, pos // page] * page + pos % page).reshape(-1).to(DEV)
        for name, pool in (("K", T.kc[l]), ("V", T.vc[l])):
            got = pool.view(-1, 8, 128)[rows].view(len(seats), k + R, 8, 128).cpu()
            ref = torch.from_numpy(gold[f"{name}{l}"].astype(np.float32))
            e_pre, e_new = _rel(got[:, :k], ref[:, :k]), _rel(got[:, k:], ref[:, k:])
            assert e_pre < tol and e_new < tol, f"{name}{l}: prefix rows {e_pre:.2e}, new rows {e_new:.2e}"
    assert np.array_equal(T.pos.cpu().numpy(), gold["pos"])
    assert torch.equal(T.x_in[seats.to(DEV)].float().cpu(), torch.from_numpy(gold["x_in"]))
    assert torch.equal(T.trail[seats.to(DEV)].float().cpu(), torch.from_numpy(gold["trail"]))
    assert np.array_equal(T.trail_len[seats.to(DEV)].cpu().numpy(), gold["trail_len"])
    assert not T.seen[seats.to(DEV)].any() and (T.ngen[seats.to(DEV)] == 0).all()
