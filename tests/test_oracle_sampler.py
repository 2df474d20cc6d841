"""CPU: the sampler oracle against the reference's own codebook-0 processing and greedy sampling
(tests/golden/sampler.npz from Talker._cb0_logits + sample_topk, engine/talker.py:90-94, engine/ops.py:68-76), the
Philox4x32-10 known-answer vectors, and the oracle's own draws against the softmax they sample from."""
import os

import numpy as np
import pytest
import torch

import make_golden as mg
from oracle import sampler as OS
from q3attn import synth


@pytest.mark.parametrize("seed", [1, 2])
def test_processing_matches_reference(golden_dir, seed):
    g = np.load(os.path.join(golden_dir, "sampler.npz"))
    d = synth.sampler_case(seed)
    assert str(g[f"s{seed}_digest"]) == mg.digest(d["logits"], d["seen"], d["seat"], d["ngen"]), "input generator drifted"
    lg = OS.process_logits(d["logits"], d["seen"], d["seat"], d["rep"], d["suppress"], d["ngen"], d["min_new"], d["eos"])
    ref = torch.from_numpy(g[f"s{seed}_processed"])
    assert torch.equal(lg, ref)
    assert torch.isinf(ref).any(), "the case exercises the suppress row / EOS mask"


@pytest.mark.parametrize("seed", [1, 2])
def test_greedy_matches_reference(golden_dir, seed):
    g = np.load(os.path.join(golden_dir, "sampler.npz"))
    lg = torch.from_numpy(g[f"s{seed}_processed"])
    ids, _ = OS.sample(lg, 1, 0.9, 0, 0)
    ref = g[f"s{seed}_greedy"]
    # equal ids, or (an exact tie at the top) the same value
    for b in range(lg.shape[0]):
        assert ids[b] == ref[b] or lg[b, ids[b]] == lg[b, ref[b]]


def test_philox_known_answers():
    """Philox4x32-10 known-answer vectors of its published reference implementation."""
    assert OS.philox4x32_10((0, 0, 0, 0), (0, 0)) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)
    f = 0xFFFFFFFF
    assert OS.philox4x32_10((f, f, f, f), (f, f)) == (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)
    assert OS.philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0)) == \
        (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)


def test_oracle_draws_follow_the_softmax():
    """Over many launch indices, the oracle's picks for one row match softmax(top-k / T) within 4 sigma."""
    lg = torch.tensor([[2.0, 1.0, 0.5, 0.0, -1.0, -3.0, float("-inf"), 1.0]])
    k, T, n = 5, 0.9, 4000
    counts = np.zeros(lg.shape[1])
    for launch in range(n):
        ids, _ = OS.sample(lg, k, T, 1234, launch)
        counts[ids[0]] += 1
    order = [0, 1, 7, 2, 3]                                   # value desc, index asc
    v = lg[0, order].double().numpy()
    p = np.exp((v - v[0]) / T)
    p /= p.sum()
    for j, i in enumerate(order):
        sd = np.sqrt(n * p[j] * (1 - p[j]))
        assert abs(counts[i] - n * p[j]) < 4 * sd + 1, (i, counts[i], n * p[j])
    assert counts[[4, 5, 6]].sum() == 0                     # outside the top k


def test_oracle_ties_at_the_kth_value_take_the_lowest_indices():
    """Winners are ranked by (value desc, index asc): among keys equal to the k-th largest value only the lowest
    indices enter the draw (the rule the GPU sampler follows)."""
    lg = torch.full((1, 40), -5.0)
    lg[0, 7] = 5.0
    lg[0, [2, 9, 20, 33]] = 3.0                  # k = 3: index 7, then 2 and 9 of the tied threes
    seen = set()
    for launch in range(200):
        ids, _ = OS.sample(lg, 3, 1e6, 11, launch)   # a huge temperature: every winner is about equally likely
        seen.add(int(ids[0]))
    assert seen == {7, 2, 9}
    ids, _ = OS.sample(lg, 1, 1.0, 11, 0)
    assert int(ids[0]) == 7
    flat = torch.zeros((1, 16))
    ids, _ = OS.sample(flat, 1, 1.0, 11, 0)
    assert int(ids[0]) == 0                       # equal maxima: the lowest index
