"""Output comparison with the prologue's FP32 rounding band (test infrastructure).

The north-star bar is 1 BF16 ulp against the ``native`` backend. One effect
makes a literal 1-ulp bound unattainable for any implementation whose sum of
squares is accumulated in a different order (a different CPU ISA, the CUDA
``native`` path, or a kernel): an output of the rotation is a difference
y1*cos - y2*sin of two products; when they nearly cancel, the FP32 rounding of
r = 1/sqrt(mean(x^2)+eps) (order-dependent in its last bit) moves the tiny
result by several ulps of itself. So an element passes when it is within
``max_ulp`` ulps, OR its absolute error is within ``band`` times the magnitude
m = |y1*cos| + |y2*sin| (times exp(scale) for Q) of the terms it was formed
from -- i.e. within FP32 rounding of the inputs to the cancellation.
"""
import torch

from .native import _broadcast_tables

DEFAULT_BAND = 2.0 ** -20  # 16 FP32 ulps of the term magnitude


def term_magnitudes(q, k, rmsnorm_weight, scales, sin, cos, eps=1e-5):
    """FP64 |y1 cos| + |y2 sin| per output element (Q includes exp(scale)), CPU tensors."""
    sin, cos, scale = _broadcast_tables(q, sin.double(), cos.double(), scales.double())
    outs = []
    for t, x in enumerate((q, k)):
        x = x.double()
        r = torch.rsqrt(x.square().mean(-1, keepdim=True) + eps)
        y = (x * r * rmsnorm_weight[t].double()).abs()
        a, b = y.chunk(2, dim=-1)
        m = torch.cat((a * cos.abs() + b * sin.abs(), b * cos.abs() + a * sin.abs()), dim=-1)
        if t == 0:
            m = m * scale.exp()
        outs.append(m)
    return tuple(outs)


def _ulps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    def ordered(t):
        if t.dtype in (torch.bfloat16, torch.float16):
            bits = t.contiguous().view(torch.int16).to(torch.int64)
            return torch.where(bits < 0, -(bits & 0x7FFF), bits)
        bits = t.contiguous().view(torch.int32).to(torch.int64)
        return torch.where(bits < 0, -(bits & 0x7FFFFFFF), bits)
    return (ordered(a) - ordered(b)).abs()


def check_outputs(got, ref, magnitude, max_ulp=1, band=DEFAULT_BAND):
    """Returns (ok, stats) for one output tensor (same dtype/shape; any device)."""
    got = got.detach()
    ref = ref.detach().to(got.device)
    magnitude = magnitude.to(got.device)
    ulps = _ulps(got, ref)
    absdiff = (got.double() - ref.double()).abs()
    in_band = absdiff <= band * magnitude.to(absdiff.dtype)
    ok_elem = (ulps <= max_ulp) | in_band
    stats = {
        "elements": got.numel(),
        "exact_frac": float((ulps == 0).double().mean()) if got.numel() else 1.0,
        "max_ulp": int(ulps.max()) if got.numel() else 0,
        "beyond_ulp_in_band": int(((ulps > max_ulp) & in_band).sum()),
        "failures": int((~ok_elem).sum()),
    }
    return stats["failures"] == 0, stats
