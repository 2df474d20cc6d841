"""fp32 CPU restatement of the reference's attention hot path (test infrastructure only; see oracle/__init__.py).

Every function cites the reference lines it restates. Tensors may be bf16 on input; all arithmetic is fp32.
"""
import torch

NEG = float("-inf")


# --------------------------------------------------------------------------- page placement
def slot_of(block_table: torch.Tensor, seat: int, pos: int, page: int) -> int:
    """Flat row index of token ``pos`` of ``seat`` in a pool viewed as [num_pages*page, nkv, hd].

    The reference writes the token at ``seat*seat_len + pos`` (engine/talker.py:109) into pages of 256 tokens whose table
    is the identity ``seat_pages[s, j] = s*P + j`` (engine/talker.py:42); through a general block table that is
    ``block_table[seat, pos // page] * page + pos % page``, and the two agree for the identity table."""
    return int(block_table[seat, pos // page]) * page + pos % page


def append_paged(k_pool, v_pool, k_new, v_new, positions, block_table):
    """In-place append of one token per seat (engine/talker.py:72-73: ``kc[l].view(-1,nkv,hd).index_copy_(0, slot, k)``).
    k_pool/v_pool [num_pages, page, nkv, hd]; k_new/v_new [B, nkv, hd]; positions [B] (token index of the new row)."""
    page = k_pool.shape[1]
    slots = torch.tensor([slot_of(block_table, b, int(positions[b]), page) for b in range(k_new.shape[0])], dtype=torch.int64)
    append_slots(k_pool, v_pool, k_new, v_new, slots)
    return slots


def append_slots(k_pool, v_pool, k_rows, v_rows, slots):
    """Flat-slot row write, exactly ``Tensor.index_copy_(0, slot, rows)`` on the pool viewed as rows
    (engine/talker.py:72-73, 161-162; engine/arrivals.py:144-145)."""
    nkv, hd = k_pool.shape[-2], k_pool.shape[-1]
    k_pool.view(-1, nkv, hd).index_copy_(0, slots.to(torch.int64), k_rows.to(k_pool.dtype))
    v_pool.view(-1, nkv, hd).index_copy_(0, slots.to(torch.int64), v_rows.to(v_pool.dtype))


def gather_seat(pool, block_table_row, n: int):
    """Contiguous [n, nkv, hd] fp32 copy of a seat's first n tokens, gathered through its block-table row."""
    page = pool.shape[1]
    npg = (n + page - 1) // page
    pages = pool[block_table_row[:npg].to(torch.int64)]          # [npg, page, nkv, hd]
    return pages.reshape(-1, pool.shape[2], pool.shape[3])[:n].float()


# --------------------------------------------------------------------------- decode
def decode_attention(q, k_pool, v_pool, seqlens, block_table, scale):
    """Paged decode attention, one query token per seat.

    Restates Talker._attn_ref (engine/talker.py:82-88): for seat b the keys 0..ctx-1 are taken, the query is viewed as
    [nkv, nh//nkv, hd] (GQA: q head h reads KV head h // 2), ``softmax(q k^T * scale) v`` in fp32. The reference reads a
    contiguous slice (identity pages); here the slice is gathered through ``block_table`` first, which is the same data
    for the identity table. q [B, nh, hd] -> [B, nh, hd] fp32."""
    B, nh, hd = q.shape
    nkv = k_pool.shape[2]
    out = []
    for b in range(B):
        n = int(seqlens[b])
        if n == 0:                                   # no keys: zeros (flash-attn writes 0 for an empty cache)
            out.append(torch.zeros(nh, hd))
            continue
        k = gather_seat(k_pool, block_table[b], n).transpose(0, 1)   # [nkv, n, hd]
        v = gather_seat(v_pool, block_table[b], n).transpose(0, 1)
        a = torch.matmul(q[b].float().view(nkv, nh // nkv, hd), k.transpose(-1, -2)) * scale
        out.append(torch.matmul(torch.softmax(a, dim=-1), v).reshape(nh, hd))
    return torch.stack(out, 0)


def decode_step(q, k_new, v_new, k_pool, v_pool, cache_seqlens, block_table, scale):
    """Append-then-attend, the order of engine/talker.py:72-77: the new K/V row of seat b is written at position
    ``cache_seqlens[b]`` and the query attends over cache_seqlens[b] + 1 tokens (so it sees itself). Mutates the pools."""
    append_paged(k_pool, v_pool, k_new, v_new, cache_seqlens, block_table)
    return decode_attention(q, k_pool, v_pool, cache_seqlens.to(torch.int64) + 1, block_table, scale)


# --------------------------------------------------------------------------- prefill
def prefill_prefix(q, K, V, scale):
    """Bottom-right causal attention of R new queries over n = k + R keys (k cached prefix + the R new ones).

    Restates FastAdmit._attn_ref (engine/arrivals.py:125-131): mask ``full((R, n), -inf).triu(n - R + 1)``; query i
    sees the prefix and new keys <= i. q [S, R, nh, hd], K/V [S, n, nkv, hd] -> [S, R, nh, hd] fp32. With k = 0 it is
    the plain causal prefill of engine/talker.py:165-167."""
    S, R, nh, hd = q.shape
    n, nkv = K.shape[1], K.shape[2]
    m = torch.full((R, n), NEG).triu(n - R + 1)
    qh = q.float().permute(0, 2, 1, 3).reshape(S, nkv, nh // nkv, R, hd)
    Kh = K.float().permute(0, 2, 1, 3)[:, :, None]
    Vh = V.float().permute(0, 2, 1, 3)[:, :, None]
    a = torch.matmul(qh, Kh.transpose(-1, -2)) * scale + m
    return torch.matmul(torch.softmax(a, dim=-1), Vh).reshape(S, nh, R, hd).permute(0, 2, 1, 3)


def prefill_varlen(q, k, v, cu_seqlens, scale, k_prefix=None, v_prefix=None, cu_prefix=None):
    """Packed varlen causal prefill (the call at engine/talker.py:169, whose fp32 twin is engine/talker.py:163-167),
    one sequence at a time; with a prefix, sequence i attends to its cached prefix first (engine/arrivals.py:148).
    q [T, nh, hd], k/v [T, nkv, hd] -> [T, nh, hd] fp32."""
    out = torch.zeros(q.shape[0], q.shape[1], q.shape[2])
    for i in range(cu_seqlens.numel() - 1):
        a, b = int(cu_seqlens[i]), int(cu_seqlens[i + 1])
        if b == a:
            continue
        K, V = k[a:b], v[a:b]
        if k_prefix is not None:
            pa, pb = int(cu_prefix[i]), int(cu_prefix[i + 1])
            K = torch.cat([k_prefix[pa:pb], K], 0)
            V = torch.cat([v_prefix[pa:pb], V], 0)
        out[a:b] = prefill_prefix(q[a:b][None], K[None], V[None], scale)[0]
    return out


# --------------------------------------------------------------------------- code predictor
def cp_mask(dtype=torch.float32):
    """The additive causal mask of engine/code_predictor.py:22-23 (row p: slots > p are -inf)."""
    return torch.full((16, 16), NEG).triu(1).to(dtype)


def cp_attention(q, K, V, n_live, scale):
    """Code-predictor attention of one step: the expression of engine/code_predictor.py:46-47 in fp32, i.e.
    ``softmax(q.view(B,8,2,128) @ K^T * scale + mask[p]) @ V`` with p = n_live - 1 (slots >= n_live masked; they
    carry no weight, which is also what engine/cp_attn.py:21-24 computes by masked loads).
    q [B, 16, 128] or [B, 2048]; K/V [B, 8, 16, 128] -> [B, 2048] fp32."""
    B = q.shape[0]
    nkv, S, hd = K.shape[1], K.shape[2], K.shape[3]
    att = torch.matmul(q.float().reshape(B, nkv, -1, hd), K.float().transpose(-1, -2)) * scale + cp_mask()[n_live - 1, :S]
    return torch.matmul(torch.softmax(att, dim=-1), V.float()).reshape(B, -1)


def cp_step(q, k_new, v_new, K, V, p, scale):
    """Slot-p append then attention over p+1 slots: engine/code_predictor.py:58 (``K.index_copy_(2, [p], k)``) followed
    by the _post attention (engine/code_predictor.py:46-47). Mutates K, V."""
    K[:, :, p] = k_new.to(K.dtype)
    V[:, :, p] = v_new.to(V.dtype)
    return cp_attention(q, K, V, p + 1, scale)
