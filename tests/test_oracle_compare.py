"""The output comparator itself: it must catch a planted 2-ulp error on a
non-cancelling element and accept rounding-band differences (CPU only)."""
import torch

from oracle import check_outputs, native_forward, term_magnitudes


def _case():
    g = torch.Generator().manual_seed(5)
    q = torch.randn(64, 4, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(64, 4, 64, generator=g).to(torch.bfloat16)
    w = 1 + 0.2 * torch.randn(2, 1, 64, generator=g)
    s = 0.1 * torch.randn(4, 1, 1, generator=g)
    ang = torch.randn(64, 32, generator=g)
    return q, k, w, s, ang.sin(), ang.cos()


def test_identical_outputs_pass():
    args = _case()
    out = native_forward(*args)
    mags = term_magnitudes(*args)
    for o, m in zip(out, mags):
        ok, stats = check_outputs(o, o.clone(), m)
        assert ok and stats["exact_frac"] == 1.0


def test_planted_two_ulp_error_is_caught():
    args = _case()
    out = native_forward(*args)
    mags = term_magnitudes(*args)
    bad = out[0].clone()
    flat = bad.view(-1).view(torch.int16)
    i = int(out[0].float().abs().view(-1).argmax())  # largest element: no cancellation
    flat[i] += 2
    ok, stats = check_outputs(bad, out[0], mags[0])
    assert not ok and stats["failures"] == 1 and stats["max_ulp"] == 2


def test_one_ulp_is_accepted():
    args = _case()
    out = native_forward(*args)
    mags = term_magnitudes(*args)
    bad = out[1].clone()
    bad.view(-1).view(torch.int16)[7] += 1
    ok, stats = check_outputs(bad, out[1], mags[1])
    assert ok and stats["max_ulp"] == 1
