"""Parity of the CUDA prologue (through the C ABI) with the reference and the oracle.

* Golden cases: the reference's own native outputs/gradients (tests/golden).
* Oracle cases: the CPU restatement of the native backend on the same seeded
  inputs, over layouts, dtypes, head dims, head counts and alignments.
* Full-size properties at the benchmark configurations: sampled-row parity
  (rows are independent), parameter gradients against an FP32 torch
  formulation, and bit-identical results run to run.

Bars: Q/K outputs within 1 ulp of the input dtype (north-star: 1 BF16 ulp),
except where the rotation's two products nearly cancel, where the error must
stay within 2^-20 of the magnitude of the terms (oracle/compare.py); more than
99% of elements must match bit for bit. FP32 outputs: rtol/atol 2e-6.
d rmsnorm_weight / d scales within 1e-3 relative error; dq/dk within the
reference tests' BF16 tolerance (atol/rtol 1e-2, tests/test_frontend_api.py:62-64)
and 5e-3 relative L2 error.
"""
import math

import pytest
import torch

from flash_attn_prologue_b200 import prepare_backend, qknorm_rope_scale
from oracle import check_outputs, native_forward, native_forward_backward, term_magnitudes
from tests._util import rel_err

pytestmark = pytest.mark.gpu

GOLDEN_NAMES = sorted(__import__("tests.golden", fromlist=["x"]).load_golden())


def _cuda_args(args):
    return [t.detach().cuda().requires_grad_(i < 4) for i, t in enumerate(args)]


def _restride_like(x: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    return torch.empty_strided(like.shape, like.stride(), dtype=x.dtype, device=like.device).copy_(x)


def _check_outputs(out, ref, dtype, inputs, eps=1e-5):
    """1 ulp, or the FP32 rounding band of a near-cancelling rotation (oracle.compare)."""
    mags = term_magnitudes(*inputs, eps=eps)
    for got, exp, mag, nm in zip(out, ref, mags, ("q_out", "k_out")):
        if dtype == torch.float32:
            torch.testing.assert_close(got.detach().cpu(), exp.cpu(), rtol=2e-6, atol=2e-6, msg=nm)
            continue
        ok, stats = check_outputs(got, exp, mag)
        assert ok, (nm, stats)
        assert stats["exact_frac"] > 0.99, (nm, stats)


def _check_grads(grads, ref, dtype):
    for got, exp, nm in zip(grads[:2], ref[:2], ("dq", "dk")):
        got = got.detach().cpu()
        if dtype == torch.float32:
            torch.testing.assert_close(got, exp, rtol=1e-4, atol=1e-5, msg=nm)
        else:
            torch.testing.assert_close(got.float(), exp.float(), rtol=1e-2, atol=1e-2, msg=nm)
            assert rel_err(got, exp) < 5e-3, nm
    assert rel_err(grads[2].detach().cpu(), ref[2]) < 1e-3, "dw"
    assert rel_err(grads[3].detach().cpu(), ref[3]) < 1e-3, "ds"


@pytest.mark.parametrize("name", GOLDEN_NAMES)
def test_golden_cases(golden, name):
    case = golden[name]
    prepare_backend("cute")
    args = _cuda_args(case.args("cuda"))
    out = qknorm_rope_scale(*args, case.eps, backend="cute")
    _check_outputs(out, (case.q_out, case.k_out), case.dtype, case.args("cpu"), case.eps)
    grads = torch.autograd.grad(out, args[:4], (case.gq.cuda(), case.gk.cuda()))
    _check_grads(grads, (case.dq, case.dk, case.dw, case.ds), case.dtype)


def _inputs(shape, d, h, dtype=torch.bfloat16, seed=0, dense_tables=None, theta=10000.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(shape, generator=g).to(dtype)
    k = torch.randn(shape, generator=g).to(dtype)
    w = 1 + 0.2 * torch.randn(2, 1, d, generator=g)
    s = 0.2 * torch.randn(h, 1, 1, generator=g) - math.log(d) / 2
    n = shape[0] if len(shape) == 3 else shape[2]
    tshape = (n, d // 2) if dense_tables is None else dense_tables
    ang = torch.randn(tshape, generator=g) * 3
    return q, k, w, s, ang.sin(), ang.cos()


def _compare_with_oracle(q, k, w, s, sin, cos, eps=1e-5, backward=True, seed=1):
    prepare_backend("cute")
    cpu = [t.detach().cpu() for t in (q, k, w, s, sin, cos)]
    g = torch.Generator().manual_seed(seed)
    gq = torch.randn(q.shape, generator=g).to(q.dtype)
    gk = torch.randn(k.shape, generator=g).to(k.dtype)
    ref_out, ref_grads = native_forward_backward(*cpu, gq, gk, eps=eps)
    args = [t.detach().requires_grad_(i < 4) for i, t in enumerate((q, k, w, s, sin, cos))]
    out = qknorm_rope_scale(*args, eps, backend="cute")
    _check_outputs(out, ref_out, q.dtype, cpu, eps)
    if backward:
        grads = torch.autograd.grad(out, args[:4], (gq.to(q.device), gk.to(q.device)))
        _check_grads(grads, ref_grads, q.dtype)


@pytest.mark.parametrize("d", [32, 64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_packed_dims_dtypes(d, dtype):
    args = _inputs((200, 6, d), d, 6, dtype, seed=d)
    _compare_with_oracle(*[t.cuda() for t in args])


@pytest.mark.parametrize("t", [1, 2, 63, 65, 129])
@pytest.mark.parametrize("d", [32, 64, 128])
@pytest.mark.parametrize("h", [1, 3])
def test_tiny_odd_token_counts(t, d, h):
    """Ragged tiles: token counts around the tile edges, one or three heads, fwd and bwd."""
    args = _inputs((t, h, d), d, h, seed=t * 7 + d + h)
    _compare_with_oracle(*[a.cuda() for a in args])
    dense = _inputs((2, h, t, d), d, h, seed=t + d, dense_tables=(2, t, d // 2))
    _compare_with_oracle(*[a.cuda() for a in dense])


@pytest.mark.parametrize("d", [32, 64, 128, 256])
@pytest.mark.parametrize("h", [1, 3, 8, 12, 32])
def test_dense_heads(d, h):
    args = list(_inputs((2, h, 77, d), d, h, seed=h * d, dense_tables=(2, 77, d // 2)))
    _compare_with_oracle(*[t.cuda() for t in args])


@pytest.mark.parametrize("h", [1, 5, 16, 48])
def test_packed_qkv_buffer_views(h):
    """q/k as strided views of one fused [T, 3, H, D] buffer (read in place)."""
    d, t = 64, 333
    g = torch.Generator().manual_seed(h)
    buf = torch.randn(t, 3, h, d, generator=g).to(torch.bfloat16).cuda()
    q, k = buf[:, 0], buf[:, 1]
    _, _, w, s, sin, cos = _inputs((t, h, d), d, h, seed=h + 1)
    _compare_with_oracle(q, k, w.cuda(), s.cuda(), sin.cuda(), cos.cuda())


def test_dense_from_bnhd_transpose():
    """Dense [B,H,N,D] views of a [B,N,H,D] buffer (heads inner, B > 1)."""
    d, h = 128, 8
    base = torch.randn(3, 50, h, d).to(torch.bfloat16).cuda()
    q = base.transpose(1, 2)
    k = torch.randn(3, 50, h, d).to(torch.bfloat16).cuda().transpose(1, 2)
    _, _, w, s, sin, cos = _inputs((50, h, d), d, h, seed=3)
    _compare_with_oracle(q, k, w.cuda(), s.cuda(), sin.cuda(), cos.cuda())


@pytest.mark.parametrize("offset", [1, 3, 8])
def test_misaligned_storage_offsets(offset):
    """Views whose rows are not 16-byte aligned take the element-wise path."""
    d, h, t = 64, 4, 65
    q, k, w, s, sin, cos = _inputs((t, h, d), d, h, seed=offset)
    def shift(x):
        st = torch.empty(x.numel() + offset, dtype=x.dtype, device="cuda")
        v = st[offset:].view_as(x)
        v.copy_(x)
        return v
    _compare_with_oracle(shift(q.cuda()), shift(k.cuda()), w.cuda(), s.cuda(),
                         shift(sin.cuda()), shift(cos.cuda()))


def test_single_position_and_eps():
    d, h = 64, 16
    q, k, w, s, sin, cos = _inputs((1, h, d), d, h, seed=11)
    _compare_with_oracle(*[t.cuda() for t in (q, k, w, s, sin, cos)], eps=0.1)


def test_large_magnitudes_and_zeros():
    d, h, t = 64, 4, 64
    q, k, w, s, sin, cos = _inputs((t, h, d), d, h, seed=12)
    q[::3] *= 300
    k[1::5] = 0  # rms = sqrt(eps): finite, outputs exactly zero rows
    _compare_with_oracle(*[t.cuda() for t in (q, k, w, s, sin, cos)])


def test_empty_inputs_cuda():
    d, h = 32, 4
    q, k, w, s, sin, cos = _inputs((0, h, d), d, h)
    args = [t.cuda().requires_grad_(i < 4) for i, t in enumerate((q, k, w, s, sin, cos))]
    out = qknorm_rope_scale(*args, backend="cute")
    assert out[0].shape == (0, h, d)
    grads = torch.autograd.grad(out, args[:4], (torch.zeros_like(out[0]), torch.zeros_like(out[1])))
    assert grads[2].abs().sum().item() == 0 and grads[3].abs().sum().item() == 0


# ----------------------------------------------------------------------------
# Full-size benchmark configurations.

def _assert_band_budget(ok, stats):
    """Full-size bar: every element within 1 BF16 ulp or the cancellation band,
    > 99% bit-exact, and at most 1e-4 of the elements (1 in 10,000) outside
    1 ulp -- the elements the band admits must stay rare."""
    assert ok, stats
    assert stats["exact_frac"] > 0.99, stats
    assert stats["beyond_ulp_in_band"] <= 1e-4 * stats["elements"], stats


def _rope(positions, d, theta):
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64, device=positions.device) / d))
    ang = (positions.double()[:, None] * inv[None]).float()
    return ang.sin(), ang.cos()


def test_config2_full_size_sampled_rows_and_param_grads():
    """C2: packed fwd+bwd from [1,048,576, 3, 16, 64] strided views."""
    T, H, D = 1 << 20, 16, 64
    g = torch.Generator(device="cuda").manual_seed(2)
    buf = torch.randn(T, 3, H, D, generator=g, device="cuda").to(torch.bfloat16)
    q, k = buf[:, 0], buf[:, 1]
    sin, cos = _rope(torch.arange(T, device="cuda") % 4096, D, 10000.0)
    w = (1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda"))
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    gq = torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16)
    gk = torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16)
    args = [t.detach().requires_grad_(i < 4) for i, t in enumerate((q, k, w, s, sin, cos))]
    out = qknorm_rope_scale(*args, backend="cute")
    grads = torch.autograd.grad(out, args[:4], (gq, gk))
    # Sampled rows against the CPU oracle.
    idx = torch.randperm(T, generator=torch.Generator().manual_seed(0))[:4096].cuda()
    sub = [x[idx].detach().cpu() for x in (q, k)]
    ref_out, ref_grads = native_forward_backward(sub[0], sub[1], w.cpu(), s.cpu(), sin[idx].cpu(),
                                                 cos[idx].cpu(), gq[idx].cpu(), gk[idx].cpu())
    mags = term_magnitudes(sub[0], sub[1], w.cpu(), s.cpu(), sin[idx].cpu(), cos[idx].cpu())
    for got, exp, mag, nm in zip((out[0][idx], out[1][idx]), ref_out, mags, ("q_out", "k_out")):
        ok, stats = check_outputs(got.cpu(), exp, mag)
        print(f"C2 sampled {nm}: {stats}")
        _assert_band_budget(ok, stats)
    for got, exp in zip((grads[0][idx], grads[1][idx]), ref_grads[:2]):
        torch.testing.assert_close(got.cpu().float(), exp.float(), rtol=1e-2, atol=1e-2)
    # Whole-problem parameter gradients against the FP32 torch formulation.
    targs = [t.detach().requires_grad_(i < 4) for i, t in enumerate((q, k, w, s, sin, cos))]
    tout = native_forward(*targs)
    tgrads = torch.autograd.grad(tout, targs[2:4], (gq, gk))
    assert rel_err(grads[2], tgrads[0]) < 1e-3
    assert rel_err(grads[3], tgrads[1]) < 1e-3


def test_config3_full_size_dense():
    """C3: dense [8, 32, 8192, 128] forward, sin/cos [S, 64] broadcast over batch."""
    B, H, S, D = 8, 32, 8192, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(B, H, S, D, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, H, S, D, generator=g, device="cuda").to(torch.bfloat16)
    sin, cos = _rope(torch.arange(S, device="cuda"), D, 500000.0)
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = torch.full((H, 1, 1), math.log(1 / math.sqrt(D)), device="cuda")
    out = qknorm_rope_scale(q, k, w, s, sin, cos, backend="cute")
    ref = native_forward(q, k, w, s, sin, cos)  # FP32 torch formulation on the GPU
    mags = term_magnitudes(q, k, w, s, sin, cos)
    for got, exp, mag, nm in zip(out, ref, mags, ("q_out", "k_out")):
        ok, stats = check_outputs(got, exp, mag)
        print(f"C3 full {nm}: {stats}")
        _assert_band_budget(ok, stats)


def test_backward_bit_reproducible():
    """C4-shaped backward twice: dq, dk, dw, ds bit-identical (fixed-order reduction)."""
    T, H, D = 262144, 8, 64
    g = torch.Generator(device="cuda").manual_seed(4)
    q, k, gq, gk = (torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16)
                    for _ in range(4))
    sin, cos = _rope(torch.arange(T, device="cuda"), D, 10000.0)
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    op = torch.ops.flash_prologue.qknorm_rope_scale_cute_backward
    q4, k4 = q.permute(1, 0, 2)[None], k.permute(1, 0, 2)[None]
    g4q, g4k = gq.permute(1, 0, 2)[None], gk.permute(1, 0, 2)[None]
    s4 = sin[None, None].expand(1, 1, T, D // 2)
    c4 = cos[None, None].expand(1, 1, T, D // 2)
    prepare_backend("cute")
    first = op(q4, k4, w, s, s4, c4, g4q, g4k, 1e-5)
    for _ in range(3):
        again = op(q4, k4, w, s, s4, c4, g4q, g4k, 1e-5)
        for a, b in zip(first, again):
            assert torch.equal(a, b)


# ----------------------------------------------------------------------------
# The kernel paths (TMA pipeline with TMA-stored or lane-stored outputs, and the
# register path) compute the same per-row arithmetic: outputs and dq/dk must be
# bit-identical; the parameter gradients of the register path differ only in
# the (fixed) grouping of their partial sums, and the two TMA store forms share
# the grid, so theirs are bit-identical too.

PATH_MODES = (0, 1, 2, 3)  # automatic, register path, TMA stores forced, lane stores forced


def _run_both_paths(args, gq, gk):
    from flash_attn_prologue_b200 import _lib
    results = []
    try:
        for mode in PATH_MODES:
            _lib.set_path(mode)
            a = [t.detach().requires_grad_(i < 4) for i, t in enumerate(args)]
            out = qknorm_rope_scale(*a, backend="cute")
            grads = torch.autograd.grad(out, a[:4], (gq, gk))
            results.append((out, grads))
    finally:
        _lib.set_path(0)
    assert _lib.device_error(reset=True) == 0
    return results


@pytest.mark.parametrize("layout", ["qkv_packed", "packed", "dense"])
@pytest.mark.parametrize("d", [32, 64, 128, 256])
def test_bulk_copy_and_register_paths_agree(layout, d):
    h, t = 8, 300
    g = torch.Generator(device="cuda").manual_seed(d)
    if layout == "qkv_packed":
        buf = torch.randn(t, 3, h, d, generator=g, device="cuda").to(torch.bfloat16)
        q, k = buf[:, 0], buf[:, 1]
        tab = (t, d // 2)
    elif layout == "packed":
        q, k = (torch.randn(t, h, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(2))
        tab = (t, d // 2)
    else:
        q, k = (torch.randn(2, h, t, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(2))
        tab = (2, t, d // 2)
    ang = torch.randn(tab, generator=g, device="cuda")
    w = 1 + 0.2 * torch.randn(2, 1, d, generator=g, device="cuda")
    s = 0.2 * torch.randn(h, 1, 1, generator=g, device="cuda")
    gq = torch.randn(q.shape, generator=g, device="cuda").to(torch.bfloat16)
    gk = torch.randn(k.shape, generator=g, device="cuda").to(torch.bfloat16)
    res = _run_both_paths((q, k, w, s, ang.sin(), ang.cos()), gq, gk)
    o0, g0 = res[0]
    for mode, (o1, g1) in zip(PATH_MODES[1:], res[1:]):
        assert torch.equal(o0[0], o1[0]) and torch.equal(o0[1], o1[1]), mode
        assert torch.equal(g0[0], g1[0]) and torch.equal(g0[1], g1[1]), mode
        if mode == 1:
            assert rel_err(g0[2], g1[2]) < 1e-5 and rel_err(g0[3], g1[3]) < 1e-5
        else:
            assert torch.equal(g0[2], g1[2]) and torch.equal(g0[3], g1[3]), mode


@pytest.mark.parametrize("d", [64, 128])
def test_broadcast_upstream_gradients(d):
    """Upstream gradients broadcast along tokens (stride 0, e.g. the gradient of a
    sum over tokens) are read in place and give the bits of the materialised
    gradient; the partially broadcast ones are read by the TMA path's fallback."""
    h, t = 4, 200
    g = torch.Generator(device="cuda").manual_seed(21 + d)
    q, k = (torch.randn(t, h, d, generator=g, device="cuda").to(torch.bfloat16) for _ in range(2))
    ang = torch.randn(t, d // 2, generator=g, device="cuda")
    w = 1 + 0.2 * torch.randn(2, 1, d, generator=g, device="cuda")
    s = 0.2 * torch.randn(h, 1, 1, generator=g, device="cuda")
    args = (q, k, w, s, ang.sin(), ang.cos())
    gq_row = torch.randn(1, h, d, generator=g, device="cuda").to(torch.bfloat16)
    gk_row = torch.randn(1, h, d, generator=g, device="cuda").to(torch.bfloat16)
    for gq, gk in ((gq_row.expand(t, h, d), gk_row.expand(t, h, d)),
                   (gq_row[:, :1].expand(t, h, d), gk_row[:, :1].expand(t, h, d))):
        got, ref = [], []
        for grads, sink in (((gq, gk), got), ((gq.contiguous(), gk.contiguous()), ref)):
            a = [x.detach().requires_grad_(i < 4) for i, x in enumerate(args)]
            out = qknorm_rope_scale(*a, backend="cute")
            sink.extend(torch.autograd.grad(out, a[:4], grads))
        assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
        assert rel_err(got[2], ref[2]) < 1e-5 and rel_err(got[3], ref[3]) < 1e-5
    from flash_attn_prologue_b200 import _lib
    assert _lib.device_error(reset=True) == 0


def test_no_device_wait_timeouts():
    from flash_attn_prologue_b200 import _lib
    assert _lib.device_error(reset=True) == 0


def test_bounded_wait_timeout_is_reported_and_context_survives():
    """Failure detection on the GPU: a wait that nothing completes gives up after
    its bound, the host reads the error word, and the next launches are correct."""
    from flash_attn_prologue_b200 import _lib
    prepare_backend("cute")
    _lib.device_error(reset=True)
    _lib.selftest_wait_timeout(4096)
    torch.cuda.synchronize()
    assert _lib.device_error(reset=True) == 1
    assert _lib.device_error(reset=True) == 0
    args = _cuda_args(_inputs((2, 4, 33, 64), 64, 4, seed=77))
    out = qknorm_rope_scale(*args, backend="cute")
    torch.cuda.synchronize()
    ref = native_forward(*[t.detach().cpu() for t in args])
    _check_outputs(out, ref, torch.bfloat16, [t.detach().cpu() for t in args])
    assert _lib.device_error(reset=True) == 0


def test_eager_path_equals_registered_op():
    """Plain eager calls skip the custom-op dispatch; outputs and gradients are the op's bits."""
    from flash_attn_prologue_b200.functional import _plain_eager
    args = [t.cuda() for t in _inputs((300, 8, 64), 64, 8, seed=9)]
    q, k, w, s, sin, cos = args
    assert _plain_eager(q, k, w, s, sin, cos)
    leaves = [t.detach().requires_grad_(i < 4) for i, t in enumerate(args)]
    out = qknorm_rope_scale(*leaves, backend="cute")
    g = [torch.randn_like(o) for o in out]
    grads = torch.autograd.grad(out, leaves[:4], g)
    q4, k4 = (t.detach().requires_grad_() for t in (q.permute(1, 0, 2)[None], k.permute(1, 0, 2)[None]))
    w2, s2 = w.detach().requires_grad_(), s.detach().requires_grad_()
    s4 = sin.permute(1, 0, 2)[None] if sin.ndim == 3 else sin[None, None]
    c4 = cos.permute(1, 0, 2)[None] if cos.ndim == 3 else cos[None, None]
    ref = torch.ops.flash_prologue.qknorm_rope_scale_cute(q4, k4, w2, s2, s4, c4, 1e-5)
    rgrads = torch.autograd.grad(ref, (q4, k4, w2, s2), [t.permute(1, 0, 2)[None] for t in g])
    assert torch.equal(out[0], ref[0].squeeze(0).permute(1, 0, 2))
    assert torch.equal(out[1], ref[1].squeeze(0).permute(1, 0, 2))
    assert torch.equal(grads[0], rgrads[0].squeeze(0).permute(1, 0, 2))
    assert torch.equal(grads[1], rgrads[1].squeeze(0).permute(1, 0, 2))
    assert torch.equal(grads[2], rgrads[2]) and torch.equal(grads[3], rgrads[3])
