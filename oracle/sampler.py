"""CPU restatement of the frame's sampling (test infrastructure only; see oracle/__init__.py).

  process_logits   engine/talker.py:90-94   repetition penalty over seen[seat], + suppress row, EOS masked while
                                            ngen[seat] < min_new
  philox4x32_10    Philox4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw, SC 2011), the random stream of
                   q3attn.sample_topk: counter (row, launch index low, launch index high, 0), key (seed low, seed high)
  sample           engine/ops.py:68-76 (top-k, softmax(vals / temperature), one draw) with the selection order and the
                   draw the GPU sampler uses: winners ranked by (value desc, index asc), u = (philox.x >> 8) / 2^24,
                   pick = first j whose inclusive prefix sum of exp((v_j - v_0) / T) exceeds u * sum
"""
import numpy as np
import torch

NEG = float("-inf")
_M0, _M1, _W0, _W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
_U32 = 0xFFFFFFFF


def process_logits(lg, seen, seat, rep, suppress, ngen, min_new, eos):
    """engine/talker.py:92-94 on fp32 logits [B, V]; seen [S, V] bool, seat [B], ngen [S]."""
    eos_col = torch.zeros(lg.shape[1], dtype=torch.bool)
    eos_col[eos] = True
    lg = torch.where(seen[seat], torch.where(lg < 0, lg * rep, lg / rep), lg) + suppress
    return lg.masked_fill((ngen[seat] < min_new)[:, None] & eos_col[None, :], NEG)


def philox4x32_10(ctr, key):
    """Four 32-bit outputs of Philox4x32-10 for a 4-word counter and a 2-word key (python ints)."""
    c0, c1, c2, c3 = (int(x) & _U32 for x in ctr)
    k0, k1 = (int(x) & _U32 for x in key)
    for r in range(10):
        if r:
            k0, k1 = (k0 + _W0) & _U32, (k1 + _W1) & _U32
        p0, p1 = _M0 * c0, _M1 * c2
        c0, c1, c2, c3 = ((p1 >> 32) ^ c1 ^ k0) & _U32, p1 & _U32, ((p0 >> 32) ^ c3 ^ k1) & _U32, p0 & _U32
    return c0, c1, c2, c3


def uniform(seed: int, row: int, launch: int) -> float:
    x = philox4x32_10((row, launch & _U32, (launch >> 32) & _U32, 0), (seed & _U32, (seed >> 32) & _U32))[0]
    return float(np.float32(x >> 8) * np.float32(1.0 / 16777216.0))


def sample(lg, k: int, temperature: float, seed: int, launch: int):
    """ids [B] for processed logits [B, V] (fp32), plus per row the relative distance of u * sum to the nearest prefix
    boundary (tiny distances are where the GPU's fp32 sums may legitimately pick the neighbour)."""
    x = lg.numpy().astype(np.float32)
    B, V = x.shape
    ids, margin = np.zeros(B, dtype=np.int64), np.full(B, np.inf)
    for b in range(B):
        order = np.lexsort((np.arange(V), -x[b].astype(np.float64)))[:k]   # value desc, index asc (-inf last)
        if k == 1:
            ids[b] = order[0]
            continue
        v = x[b, order].astype(np.float64)
        if not np.isfinite(v[0]):
            ids[b] = order[0]
            continue
        e = np.exp((v - v[0]) / temperature)
        cum = np.cumsum(e)
        t = uniform(seed, b, launch) * cum[-1]
        j = int(np.searchsorted(cum, t, side="right"))
        j = min(j, k - 1)
        ids[b] = order[j]
        margin[b] = np.min(np.abs(cum - t)) / cum[-1]
    return ids, margin
