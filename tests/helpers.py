"""Shared checks for the tests."""
import torch

# north star tolerance for bf16 attention outputs vs the fp32-accumulated reference: max-abs 1e-2, rel 2e-2
ATOL, RTOL = 1e-2, 2e-2


def assert_close_attn(got: torch.Tensor, ref: torch.Tensor, atol: float = ATOL, rtol: float = RTOL, what: str = ""):
    g = got.detach().float().cpu()
    r = ref.detach().float().cpu()
    assert g.shape == r.shape, (g.shape, r.shape)
    assert torch.isfinite(g).all(), f"{what}: non-finite output"
    err = (g - r).abs()
    bound = atol + rtol * r.abs()
    bad = err > bound
    if bad.any():
        i = int(err.argmax())
        raise AssertionError(f"{what}: {int(bad.sum())} of {g.numel()} elements outside |d| <= {atol} + {rtol}|ref|; "
                             f"max |d| = {float(err.max()):.3e} at flat {i} (got {float(g.flatten()[i]):.5f}, "
                             f"ref {float(r.flatten()[i]):.5f})")


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.detach().cpu().contiguous(), b.detach().cpu().contiguous()
    return a.shape == b.shape and a.dtype == b.dtype and torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                                                                      b.view(torch.int16) if b.dtype == torch.bfloat16 else b)


def poison_allocator(shape, dtype=torch.bfloat16, device="cuda:0", n=4):
    """Fill and free a few blocks of the op's output size with NaN, so the caching allocator hands the op NaN-filled
    memory: an output element the kernel forgets to write then fails the comparison instead of passing on stale data."""
    ts = [torch.full(shape, float("nan"), dtype=dtype, device=device) for _ in range(n)]
    del ts
