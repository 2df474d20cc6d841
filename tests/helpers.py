"""Shared checks for the tests."""
import torch

# north star tolerance for bf16 attention outputs vs the fp32-accumulated reference, as two separate bounds:
# max-abs 1e-2 over every element, and relative error 2e-2 (||got - ref|| / ||ref||, 2-norm over the whole output)
ATOL, RTOL = 1e-2, 2e-2


def attn_errors(got: torch.Tensor, ref: torch.Tensor):
    """(max |got - ref|, ||got - ref||_2 / ||ref||_2) in fp32 on the CPU."""
    g = got.detach().float().cpu()
    r = ref.detach().float().cpu()
    d = g - r
    return float(d.abs().max()) if d.numel() else 0.0, float(d.norm() / r.norm().clamp_min(1e-30))


def assert_close_attn(got: torch.Tensor, ref: torch.Tensor, atol: float = ATOL, rtol: float = RTOL, what: str = ""):
    """Max-abs error <= atol AND relative error <= rtol, checked separately (not the combined atol + rtol*|ref|)."""
    g = got.detach().float().cpu()
    r = ref.detach().float().cpu()
    assert g.shape == r.shape, (g.shape, r.shape)
    assert torch.isfinite(g).all(), f"{what}: non-finite output"
    max_abs, rel = attn_errors(g, r)
    if max_abs > atol or rel > rtol:
        err = (g - r).abs()
        i = int(err.argmax())
        raise AssertionError(f"{what}: max |d| = {max_abs:.3e} (bound {atol}), rel = {rel:.3e} (bound {rtol}); "
                             f"worst at flat {i} (got {float(g.flatten()[i]):.5f}, ref {float(r.flatten()[i]):.5f}), "
                             f"{int((err > atol).sum())} of {g.numel()} elements above {atol}")


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.detach().cpu().contiguous(), b.detach().cpu().contiguous()
    return a.shape == b.shape and a.dtype == b.dtype and torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                                                                      b.view(torch.int16) if b.dtype == torch.bfloat16 else b)


def poison_allocator(shape, dtype=torch.bfloat16, device="cuda:0", n=4):
    """Fill and free a few blocks of the op's output size with NaN, so the caching allocator hands the op NaN-filled
    memory: an output element the kernel forgets to write then fails the comparison instead of passing on stale data."""
    ts = [torch.full(shape, float("nan"), dtype=dtype, device=device) for _ in range(n)]
    del ts
