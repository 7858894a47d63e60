"""Comparison helpers shared by the tests."""
import torch


def ordered_bits(t: torch.Tensor) -> torch.Tensor:
    """Monotone integer image of a 16/32-bit float tensor (adjacent floats differ by 1)."""
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        bits = t.view(torch.int16).to(torch.int64)
        return torch.where(bits < 0, -(bits & 0x7FFF), bits)
    bits = t.view(torch.int32).to(torch.int64)
    return torch.where(bits < 0, -(bits & 0x7FFFFFFF), bits)


def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Element-wise distance in units in the last place (same dtype tensors)."""
    assert a.dtype == b.dtype and a.shape == b.shape, (a.dtype, b.dtype, a.shape, b.shape)
    return (ordered_bits(a) - ordered_bits(b)).abs()


def assert_ulp(a, b, max_ulp=1, name=""):
    d = ulp_diff(a, b)
    worst = int(d.max()) if d.numel() else 0
    assert worst <= max_ulp, f"{name}: max ulp {worst} > {max_ulp} ({int((d > max_ulp).sum())} elements)"
    return d


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))
