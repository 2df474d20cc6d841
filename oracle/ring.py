"""CPU restatement of the streaming codec decoder's windowed ring attention (test infrastructure only; see
oracle/__init__.py): the ring-mode attention of StreamCore.forward, engine/decoder_stream.py:147-181, for one layer.

Stream b's ring holds the rotated K/V of frame f in slot f % RING. The chunk's n queries at positions pos .. pos+n-1
see ring slot j (frame qj = (pos-1) - ((pos-1-j) mod RING)) when qj >= 0 and qj >= (pos+i) - PAST, and the chunk's own
keys up to themselves; lg = [q.K_ring, q.k_new] * scale + bias, P = softmax(lg), o = P_ring.V_ring + P_new.v_new.
`emulate_fp16` adds the rounding points the reference's fp16 matmuls have (scores, P and each P.V half rounded to fp16).
"""
import torch


def ring_attention(q, k_new, v_new, K_ring, V_ring, pos, past, scale, emulate_fp16=False):
    """q / k_new / v_new [B, n, H, hd]; K_ring / V_ring [B, RING, H, hd] (each batch entry's ring); pos [B].
    Returns o [B, n, H * hd] fp32."""
    B, n, H, hd = q.shape
    RING = K_ring.shape[1]
    r = (lambda t: t.half().float()) if emulate_fp16 else (lambda t: t)
    qv = q.float().permute(0, 2, 1, 3)                                 # [B, H, n, hd]
    kv = k_new.float().permute(0, 2, 1, 3)
    vv = v_new.float().permute(0, 2, 1, 3)
    Kl = K_ring.float().permute(0, 2, 3, 1)                            # [B, H, hd, RING]
    Vl = V_ring.float().permute(0, 2, 1, 3)                            # [B, H, RING, hd]
    ar = torch.arange(n)
    pm1 = (pos.long() - 1)[:, None]
    qj = pm1 - torch.remainder(pm1 - torch.arange(RING)[None], RING)   # frame held by each slot
    a_ = (pos.long()[:, None] + ar[None])[:, :, None]
    old_ok = (qj[:, None, :] >= 0) & (qj[:, None, :] >= a_ - past)
    new_ok = (ar[None, :] <= ar[:, None])[None].expand(B, -1, -1)
    bias = torch.zeros(B, n, RING + n).masked_fill(~torch.cat((old_ok, new_ok), -1), float("-inf"))[:, None]
    lg = torch.cat((r(torch.matmul(qv, Kl)), r(torch.matmul(qv, kv.transpose(-1, -2)))), dim=-1) * scale + bias
    P = r(torch.softmax(lg, dim=-1))
    o = r(r(torch.matmul(P[..., :RING], Vl)) + r(torch.matmul(P[..., RING:], vv)))
    return o.permute(0, 2, 1, 3).reshape(B, n, H * hd)
