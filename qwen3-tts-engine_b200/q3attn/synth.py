"""Seeded synthetic workloads with the shapes of the engine's attention hot path.

Every integer layout (context lengths, page tables) is drawn on the CPU from ``torch.Generator().manual_seed(seed)`` so a
test on the GPU box and a fixture generated elsewhere see the same seats and pages. Large tensor contents for the bench
are drawn on the device from a seeded CUDA generator (their values do not change the timing).

Shapes (the engine's model family, engine/talker.py:26, engine/code_predictor.py:16):
  16 query heads, 8 KV heads (GQA group 2), head_dim 128; one token row of a page holds all 8 KV heads (2 KB in bf16).

Configurations:
  C1  4 seats, ctx U[1,256], page 16, 128-page pool, pages assigned by a seeded permutation, fp32, N(0,1).
  C2  0.6B talker decode: 28 layers, 576 seats, ctx U[200,1200] (+1 appended token), page 16, pool for 576*1216 tokens,
      shuffled page table, N(0,1)*0.5 bf16.
  C3  1.7B talker: 470 decoding seats ctx U[100,1500] + 10 seats prefilling 320-token prompts into fresh pages.
  C4  code predictor: 5 layers, 576 seats, 16-slot per-seat cache, 15 steps with n_live 2..16.
"""
from dataclasses import dataclass

import torch

NH, NKV, HD = 16, 8, 128
GROUP = NH // NKV
ROW_ELEMS = NKV * HD          # elements of one token row (all KV heads)


def cpu_gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(int(seed))


@dataclass
class PagedLayout:
    """Which physical pages each seat owns and how many tokens each seat holds."""
    ctx: torch.Tensor            # int32 [B]: tokens already in the cache (before any append)
    block_table: torch.Tensor    # int32 [B, pages_per_seat]
    page: int
    num_pages: int

    @property
    def B(self) -> int:
        return int(self.ctx.shape[0])


def paged_layout(seed: int, B: int, ctx_lo: int, ctx_hi: int, page: int, pages_per_seat: int,
                 num_pages: int | None = None) -> PagedLayout:
    """ctx ~ U[ctx_lo, ctx_hi] per seat; the page table is a seeded shuffle of the pool (seat s owns
    perm[s*pps:(s+1)*pps])."""
    g = cpu_gen(seed)
    ctx = torch.randint(ctx_lo, ctx_hi + 1, (B,), generator=g, dtype=torch.int64).to(torch.int32)
    num_pages = num_pages or B * pages_per_seat
    assert num_pages >= B * pages_per_seat
    perm = torch.randperm(num_pages, generator=g)[: B * pages_per_seat]
    bt = perm.view(B, pages_per_seat).to(torch.int32).contiguous()
    return PagedLayout(ctx=ctx, block_table=bt, page=page, num_pages=num_pages)


def c1_layout(seed: int = 1) -> PagedLayout:
    """4 seats, ctx U[1,256], page 16, a 128-page pool assigned by a seeded permutation."""
    return paged_layout(seed, B=4, ctx_lo=1, ctx_hi=256, page=16, pages_per_seat=16, num_pages=128)


def c2_layout(seed: int = 2, B: int = 576) -> PagedLayout:
    """576 seats, ctx U[200,1200], page 16, pool sized for 576*1216 tokens (76 pages per seat)."""
    return paged_layout(seed, B=B, ctx_lo=200, ctx_hi=1200, page=16, pages_per_seat=1216 // 16, num_pages=B * 1216 // 16)


def c3_layout(seed: int = 3):
    """470 decoding seats ctx U[100,1500] and 10 admitting seats prefilling 320 tokens each.
    Returns (decode layout over all 480 seats' pools, prefill seats, prompt length). The pool holds 1536 tokens per seat."""
    pps = 1536 // 16
    lay = paged_layout(seed, B=480, ctx_lo=100, ctx_hi=1500, page=16, pages_per_seat=pps)
    lay.ctx[470:] = 0                     # the admitting seats start empty and receive a 320-token chunk
    return lay, list(range(470, 480)), 320


def randn(shape, gen: torch.Generator, scale: float = 1.0, dtype=torch.float32, device="cpu") -> torch.Tensor:
    """N(0,1)*scale drawn in fp32 with ``gen`` then cast to ``dtype``."""
    if str(device).startswith("cuda") and gen.device.type == "cuda":
        x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    else:
        x = torch.randn(shape, generator=gen, dtype=torch.float32).to(device)
    if scale != 1.0:
        x.mul_(scale)
    return x.to(dtype)


def decode_case(seed: int, lay: PagedLayout, scale: float = 0.5, dtype=torch.bfloat16, device="cpu"):
    """Pool contents and the step's new q/k/v for one layer of a paged decode step, all drawn from ``seed`` on the CPU.

    Returns dict(q [B,16,128], k_new [B,8,128], v_new [B,8,128], k_pool/v_pool [num_pages, page, 8, 128])."""
    g = cpu_gen(seed + 1000)
    shp = (lay.num_pages, lay.page, NKV, HD)
    out = dict(
        q=randn((lay.B, NH, HD), g, scale, dtype, device),
        k_new=randn((lay.B, NKV, HD), g, scale, dtype, device),
        v_new=randn((lay.B, NKV, HD), g, scale, dtype, device),
        k_pool=randn(shp, g, scale, dtype, device),
        v_pool=randn(shp, g, scale, dtype, device),
    )
    return out


def cp_case(seed: int, B: int, dtype=torch.bfloat16, device="cpu", slots: int = 16):
    """Code-predictor step inputs: q [B,16,128], k/v new [B,8,128] and the per-seat 16-slot caches [B,8,16,128]
    (engine/code_predictor.py:20-21 layout for one layer), N(0,1)."""
    g = cpu_gen(seed + 2000)
    return dict(
        q=randn((B, NH, HD), g, 1.0, dtype, device),
        k_new=randn((B, NKV, HD), g, 1.0, dtype, device),
        v_new=randn((B, NKV, HD), g, 1.0, dtype, device),
        K=randn((B, NKV, slots, HD), g, 1.0, dtype, device),
        V=randn((B, NKV, slots, HD), g, 1.0, dtype, device),
    )


def prefill_case(seed: int, lens, prefix_lens=None, scale: float = 0.5, dtype=torch.bfloat16, device="cpu"):
    """Packed prompt rows for a varlen causal prefill: q [T,16,128], k/v [T,8,128] with cu_seqlens int32 [n+1].
    ``prefix_lens`` (optional) gives tokens already cached ahead of each prompt (bottom-right causal alignment)."""
    g = cpu_gen(seed + 3000)
    lens = [int(x) for x in lens]
    T = sum(lens)
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0).to(torch.int32)
    out = dict(q=randn((T, NH, HD), g, scale, dtype, device), k=randn((T, NKV, HD), g, scale, dtype, device),
               v=randn((T, NKV, HD), g, scale, dtype, device), cu_seqlens=cu.to(device), lens=lens)
    if prefix_lens is not None:
        P = sum(int(x) for x in prefix_lens)
        cp = torch.zeros(len(lens) + 1, dtype=torch.int32)
        cp[1:] = torch.cumsum(torch.tensor([int(x) for x in prefix_lens], dtype=torch.int64), 0).to(torch.int32)
        out.update(k_prefix=randn((P, NKV, HD), g, scale, dtype, device), v_prefix=randn((P, NKV, HD), g, scale, dtype, device),
                   cu_prefix=cp.to(device), prefix_lens=[int(x) for x in prefix_lens])
    return out


def sampler_case(seed: int, B: int = 24, S: int = 30, V: int = 3072, eos: int = 2150, scale: float = 3.0):
    """Inputs of one codebook-0 sampling call (engine/talker.py:90-97): bf16-representable fp32 logits [B, V], a
    `seen` table [S, V] (5% set), distinct seats [B], ngen [S] in 0..3, and the reference's suppress row (ids
    >= V - 1024 at -inf except EOS, talker.py:43)."""
    g = cpu_gen(seed + 3000)
    logits = (torch.randn(B, V, generator=g) * scale).to(torch.bfloat16).float()
    seen = torch.rand(S, V, generator=g) < 0.05
    seat = torch.randperm(S, generator=g)[:B].to(torch.int64)
    ngen = torch.randint(0, 4, (S,), generator=g, dtype=torch.int64)
    sup = torch.zeros(V)
    sup[V - 1024:] = float("-inf")
    sup[eos] = 0.0
    return dict(logits=logits, seen=seen, seat=seat, ngen=ngen, suppress=sup, eos=eos, rep=1.05, min_new=2)


def decode_bytes(ctx_after: torch.Tensor, append: bool = True) -> int:
    """Algorithmic HBM bytes of one paged decode layer: K+V read of every attended token (4096 B each), q read and o
    write (4096 B each per seat), the fused append write (4096 B per seat) and the page-table entries read."""
    c = ctx_after.to(torch.int64)
    n = int(c.numel())
    pages = int(((c + 15) // 16).sum())
    return int(4096 * int(c.sum()) + 8192 * n + (4096 * n if append else 0) + 4 * pages)


# --------------------------------------------------------------------------- device-independent K/V history
_M32 = 0xFFFFFFFF


def _mix32(x: torch.Tensor) -> torch.Tensor:
    """A 32-bit xorshift-multiply mixer on int64 tensors holding values in [0, 2^32): every product stays below 2^63
    (32-bit value x 31-bit constant), so CPU and CUDA integer arithmetic give the same bits."""
    x = x ^ (x >> 16)
    x = (x * 0x7FEB352D) & _M32
    x = x ^ (x >> 15)
    x = (x * 0x5BD1E995) & _M32
    return x ^ (x >> 16)


def history_block(seed: int, layer: int, kv: int, seats: torch.Tensor, n_rows: int, device="cpu") -> torch.Tensor:
    """Token rows 0..n_rows-1 of the K (kv = 0) or V (kv = 1) history of each seat in `seats` in one layer:
    [len(seats), n_rows, 8, 128] fp32 whose values are a pure function of (seed, layer, kv, seat, position, head, dim),
    bit-identical on the CPU and on the GPU. Each value is (a + b + c + d - 126) / 64 for four 6-bit fields of a hashed
    counter: symmetric, bell-shaped (Irwin-Hall of four uniforms), standard deviation 0.577, and exactly representable
    in bf16. This lets a fixture made by the reference on the CPU and a GPU test share a K/V history far too large to
    store."""
    seats = torch.as_tensor(seats, dtype=torch.int64, device=device).view(-1)
    key = ((int(seed) * 64 + int(layer)) * 2 + int(kv)) * 1_000_003 + seats
    s = _mix32(key & _M32)
    e = torch.arange(n_rows * ROW_ELEMS, dtype=torch.int64, device=device)
    x = _mix32((e[None, :] + s[:, None] * 0x9E37) & _M32)
    u = (x & 63) + ((x >> 6) & 63) + ((x >> 12) & 63) + ((x >> 18) & 63) - 126
    return (u.to(torch.float32) * (1.0 / 64)).view(seats.numel(), n_rows, NKV, HD)


def history_rows(seed: int, layer: int, kv: int, seat: int, n_rows: int, device="cpu") -> torch.Tensor:
    """history_block for one seat: [n_rows, 8, 128]."""
    return history_block(seed, layer, kv, torch.tensor([seat]), n_rows, device)[0]
