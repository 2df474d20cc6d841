"""GPU parity: logit processing + top-k sampling (engine/talker.py:90-94, engine/ops.py:68-76) through q3_sample_topk,
against the oracle (itself pinned to the reference in tests/test_oracle_sampler.py): greedy ids exactly; sampled ids
exactly except where u * sum lands within fp32 rounding of a prefix-sum boundary; the random stream advancing once per
launch, CUDA-graph replays included."""
import os

import numpy as np
import pytest
import torch

from helpers import bits_equal
from oracle import sampler as OS
from q3attn import synth

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def q3():
    import q3attn
    q3attn._lib.load()
    return q3attn


def _dev(d):
    return {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}


def _check_sampled(ids, ref, margin, what, tol=1e-5):
    ids = ids.cpu().numpy()
    bad = [(b, int(ids[b]), int(ref[b]), float(margin[b])) for b in range(len(ids)) if ids[b] != ref[b]]
    assert all(m < tol for *_, m in bad), f"{what}: picks differ away from a boundary: {bad[:5]}"
    assert len(bad) <= max(1, len(ids) // 100), f"{what}: {len(bad)} of {len(ids)} picks differ"


@pytest.mark.parametrize("seed", [1, 2])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_cb0_processing_and_greedy(q3, golden_dir, seed, dtype):
    d = synth.sampler_case(seed)
    g = _dev(d)
    rng = q3.SamplerRng(5, DEV)
    ids = q3.sample_topk(g["logits"].to(dtype), 0.9, 1, rng, seen=g["seen"], seat=g["seat"], rep_penalty=d["rep"],
                         bias=g["suppress"], ngen=g["ngen"], min_new=d["min_new"], eos=d["eos"])
    torch.cuda.synchronize()
    gold = np.load(os.path.join(golden_dir, "sampler.npz"))
    lg = torch.from_numpy(gold[f"s{seed}_processed"])
    ref, _ = OS.sample(lg, 1, 0.9, 5, 0)
    assert np.array_equal(ids.cpu().numpy(), ref)
    assert rng.launch_index == 1


@pytest.mark.parametrize("k,T", [(50, 0.9), (2, 1.0), (64, 0.5), (7, 2.0)])
def test_topk_sampling_follows_the_oracle_stream(q3, k, T):
    d = synth.sampler_case(3, B=96, S=128)
    g = _dev(d)
    lg = OS.process_logits(d["logits"], d["seen"], d["seat"], d["rep"], d["suppress"], d["ngen"], d["min_new"], d["eos"])
    rng = q3.SamplerRng(0x1234_5678_9ABC, DEV)
    for launch in range(3):
        ids = q3.sample_topk(g["logits"], T, k, rng, seen=g["seen"], seat=g["seat"], rep_penalty=d["rep"],
                             bias=g["suppress"], ngen=g["ngen"], min_new=d["min_new"], eos=d["eos"])
        ref, margin = OS.sample(lg, k, T, rng.seed, launch)
        _check_sampled(ids, ref, margin, f"k {k} T {T} launch {launch}")
    assert rng.launch_index == 3


def test_embedding_rows_and_plain_rows(q3):
    """No processing (the code predictor's heads, code_predictor.py:70-71): ids and the embedding rows of the ids."""
    gen = synth.cpu_gen(9)
    B, V, H = 130, 2048, 1024
    lg = synth.randn((B, V), gen, 2.0, torch.bfloat16)
    emb = synth.randn((V, H), gen, 1.0, torch.bfloat16)
    rng = q3.SamplerRng(77, DEV)
    ids, e = q3.sample_topk(lg.to(DEV), 0.9, 50, rng, emb=emb.to(DEV))
    torch.cuda.synchronize()
    ref, margin = OS.sample(lg.float(), 50, 0.9, 77, 0)
    _check_sampled(ids, ref, margin, "plain rows")
    assert bits_equal(e, emb.to(DEV)[ids])


def test_edges_ties_small_vocab_and_masked_rows(q3):
    rng = q3.SamplerRng(3, DEV)
    # all-equal row: greedy takes index 0, k = 3 draws among indices 0..2 only
    flat = torch.zeros(4, 300, device=DEV)
    assert q3.sample_topk(flat, 1.0, 1, rng).tolist() == [0, 0, 0, 0]
    ids = q3.sample_topk(flat, 1.0, 3, rng)
    assert set(ids.tolist()) <= {0, 1, 2}
    # vocab not a multiple of the block, k == vocab
    gen = synth.cpu_gen(4)
    lg = synth.randn((17, 40), gen, 1.0)
    ids = q3.sample_topk(lg.to(DEV), 1.3, 40, rng)
    ref, margin = OS.sample(lg, 40, 1.3, 3, 2)
    _check_sampled(ids, ref, margin, "k == vocab")
    # a row with every entry at -inf but one: that one is always picked, any k
    m = torch.full((3, 2500), float("-inf"))
    m[:, 2499] = 0.5
    assert q3.sample_topk(m.to(DEV), 0.9, 50, rng).tolist() == [2499] * 3
    torch.cuda.synchronize()
    assert rng.launch_index == 4


def test_ties_at_the_kth_value(q3):
    """Ties at the k-th largest value, few enough for the atomic winner placement (<= 64 equal keys): the lowest
    indices among them are the winners, whatever order the atomics placed them in."""
    gen = synth.cpu_gen(21)
    B, V, k = 40, 3000, 15
    lg = synth.randn((B, V), gen, 1.0) - 10.0                   # below every planted value
    for b in range(B):
        perm = torch.randperm(V, generator=gen)
        lg[b, perm[:10]] = 5.0                                  # 10 keys above the threshold
        lg[b, perm[10:10 + 20 + b % 30]] = 3.0                  # 20..49 keys equal to it: 5 of them are taken
    rng = q3.SamplerRng(8, DEV)
    ids = q3.sample_topk(lg.to(DEV), 1.0, k, rng)
    torch.cuda.synchronize()
    ref, margin = OS.sample(lg, k, 1.0, 8, 0)
    _check_sampled(ids, ref, margin, "ties at the k-th value")
    # greedy over rows whose maximum repeats: the lowest index of the maximum
    g1 = q3.sample_topk(lg.to(DEV), 1.0, 1, rng)
    assert g1.cpu().tolist() == [int(torch.nonzero(lg[b] == 5.0)[0]) for b in range(B)]


def test_graph_replays_advance_the_stream(q3):
    gen = synth.cpu_gen(12)
    B, V = 64, 2048
    lg = synth.randn((B, V), gen, 2.0)
    x = lg.to(DEV)
    rng = q3.SamplerRng(99, DEV)
    out = torch.empty(B, dtype=torch.int64, device=DEV)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out.copy_(q3.sample_topk(x, 0.9, 50, rng))              # launch 0, outside the graph
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            out.copy_(q3.sample_topk(x, 0.9, 50, rng))          # captured, not run
    torch.cuda.synchronize()
    assert rng.launch_index == 1
    for launch in (1, 2, 3):
        graph.replay()
        torch.cuda.synchronize()
        ref, margin = OS.sample(lg, 50, 0.9, 99, launch)
        _check_sampled(out, ref, margin, f"replay {launch}")
    assert rng.launch_index == 4
