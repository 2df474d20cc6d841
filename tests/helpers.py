"""Shared checks for the tests."""
import torch

# north star tolerance for bf16 attention outputs vs the fp32-accumulated reference, as two separate bounds:
#   max-abs 1e-2 for every element, except that no element is held closer than one bf16 step (ulp) at its own
#     magnitude: the output is bf16, and for |ref| >= 2 one bf16 step (2^-6 and up) already exceeds 1e-2, so even the
#     correctly rounded fp32 result can miss 1e-2 there; for |ref| < 2 the bound is exactly 1e-2;
#   relative error 2e-2 (||got - ref|| / ||ref||, 2-norm over the whole output).
ATOL, RTOL = 1e-2, 2e-2


def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 values at |x| (8 significant bits): 2^(floor(log2|x|) - 7); 2^-133 at zero."""
    e = torch.floor(torch.log2(x.abs().clamp_min(2.0 ** -126)))
    return torch.exp2(e - 7)


def attn_errors(got: torch.Tensor, ref: torch.Tensor, atol: float = ATOL):
    """(max |got - ref|, worst ratio of |got - ref| to its element bound max(atol, bf16 ulp of ref),
    ||got - ref||_2 / ||ref||_2), in fp32 on the CPU."""
    g = got.detach().float().cpu()
    r = ref.detach().float().cpu()
    d = (g - r).abs()
    if d.numel() == 0:
        return 0.0, 0.0, 0.0
    bound = torch.maximum(torch.full_like(r, atol), bf16_ulp(r))
    return float(d.max()), float((d / bound).max()), float((g - r).norm() / r.norm().clamp_min(1e-30))


def assert_close_attn(got: torch.Tensor, ref: torch.Tensor, atol: float = ATOL, rtol: float = RTOL, what: str = ""):
    """Max-abs bound (atol, or one bf16 ulp where that is larger) AND relative error <= rtol, checked separately (not
    the combined atol + rtol*|ref|)."""
    g = got.detach().float().cpu()
    r = ref.detach().float().cpu()
    assert g.shape == r.shape, (g.shape, r.shape)
    assert torch.isfinite(g).all(), f"{what}: non-finite output"
    max_abs, worst, rel = attn_errors(g, r, atol)
    if worst > 1.0 or rel > rtol:
        err = (g - r).abs() / torch.maximum(torch.full_like(r, atol), bf16_ulp(r))
        i = int(err.argmax())
        raise AssertionError(f"{what}: max |d| = {max_abs:.3e}, worst |d| / bound = {worst:.3f} (bound max({atol}, "
                             f"bf16 ulp)), rel = {rel:.3e} (bound {rtol}); worst at flat {i} (got "
                             f"{float(g.flatten()[i]):.5f}, ref {float(r.flatten()[i]):.5f}), "
                             f"{int((err > 1).sum())} of {g.numel()} elements above their bound")


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.detach().cpu().contiguous(), b.detach().cpu().contiguous()
    return a.shape == b.shape and a.dtype == b.dtype and torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                                                                      b.view(torch.int16) if b.dtype == torch.bfloat16 else b)


def poison_allocator(shape, dtype=torch.bfloat16, device="cuda:0", n=4):
    """Fill and free a few blocks of the op's output size with NaN, so the caching allocator hands the op NaN-filled
    memory: an output element the kernel forgets to write then fails the comparison instead of passing on stale data."""
    ts = [torch.full(shape, float("nan"), dtype=dtype, device=device) for _ in range(n)]
    del ts
