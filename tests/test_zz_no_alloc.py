"""The allocation-free backward entry point, flash_prologue_bwd_noalloc.

It serves callers that cannot allocate device memory per call (runtimes that
plan all device memory up front, host-language bindings without a device
allocator); its scratch is a static 1 MiB array inside the library. Checked
here through the C ABI against the existing entry point (flash_prologue_bwd,
reached through the flash_prologue::qknorm_rope_scale_cute_backward op), on two
calls in a row with different inputs, so nothing left in the shared scratch by
the first call can leak into the second; and for the rejection of a problem
too large for the scratch. This file is collected last, so a run that stops at
the first failure has run every other test before it.
"""
import ctypes

import pytest
import torch

from flash_attn_prologue_b200 import _lib, prepare_backend
from flash_attn_prologue_b200.fused_epilogue import _get_compact_strides
from tests._util import rel_err

pytestmark = pytest.mark.gpu


def _problem(seed, T=4096, H=8, D=64):
    g = torch.Generator(device="cuda").manual_seed(seed)
    buf = torch.randn(T, 3, H, D, generator=g, device="cuda").to(torch.bfloat16)
    q4 = buf[:, 0].permute(1, 0, 2)[None]
    k4 = buf[:, 1].permute(1, 0, 2)[None]
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    ang = torch.randn(T, D // 2, generator=g, device="cuda")
    sin, cos = ang.sin(), ang.cos()
    gq4 = torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16).permute(1, 0, 2)[None]
    gk4 = torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16).permute(1, 0, 2)[None]
    return buf, q4, k4, w, s, sin, cos, gq4, gk4


def _call_noalloc(q4, k4, w, s, sin, cos, gq4, gk4):
    """Outputs are created here (by the caller); the entry point allocates nothing."""
    B, H, N, D = q4.shape
    dq = torch.empty_strided(q4.shape, _get_compact_strides(q4.shape, q4.stride()),
                             dtype=q4.dtype, device=q4.device)
    dk = torch.empty_strided(k4.shape, _get_compact_strides(k4.shape, k4.stride()),
                             dtype=k4.dtype, device=k4.device)
    dw = torch.empty(2, 1, D, device=q4.device)
    ds = torch.empty(H, 1, 1, device=q4.device)
    table = _lib.strides3((0, sin.stride(0), sin.stride(1)))
    status = _lib.load().flash_prologue_bwd_noalloc(
        _lib.ptr(q4), _lib.strides4(q4), _lib.ptr(k4), _lib.strides4(k4),
        _lib.ptr(w), _lib.ptr(s), _lib.ptr(sin), table, _lib.ptr(cos), table,
        _lib.ptr(gq4), _lib.strides4(gq4), _lib.ptr(gk4), _lib.strides4(gk4),
        _lib.ptr(dq), _lib.strides4(dq), _lib.ptr(dk), _lib.strides4(dk),
        _lib.ptr(dw), _lib.ptr(ds), B, H, N, D, 1e-5, 0, _lib.stream_of(q4.device))
    _lib.check(status, "flash_prologue_bwd_noalloc")
    return dq, dk, dw, ds


def _call_existing(q4, k4, w, s, sin, cos, gq4, gk4):
    T, half = sin.shape
    sin4 = sin[None, None].expand(1, 1, T, half)
    cos4 = cos[None, None].expand(1, 1, T, half)
    return torch.ops.flash_prologue.qknorm_rope_scale_cute_backward(
        q4, k4, w, s, sin4, cos4, gq4, gk4, 1e-5)


def test_noalloc_backward_matches_workspace_backward_twice():
    prepare_backend("cute")
    for seed in (0, 1):  # two calls in a row, different inputs
        args = _problem(seed)[1:]
        got = _call_noalloc(*args)
        ref = _call_existing(*args)
        torch.cuda.synchronize()
        for a, b in zip(got[:2], ref[:2]):
            torch.testing.assert_close(a.float(), b.float(), rtol=1e-2, atol=1e-2)
        assert rel_err(got[2], ref[2]) < 1e-3
        assert rel_err(got[3], ref[3]) < 1e-3
    assert _lib.device_error(reset=True) == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    # D=256, H=512: (2*D + H) floats per CTA partial exceed 1 MiB at full occupancy.
    lib = _lib.load()
    s4 = _lib.strides4(torch.empty(1, 1, 1, 1))
    t3 = _lib.strides3((0, 128, 1))
    null = ctypes.c_void_p(0)
    status = lib.flash_prologue_bwd_noalloc(
        null, s4, null, s4, null, null, null, t3, null, t3, null, s4, null, s4,
        null, s4, null, s4, null, null, 1, 512, 4096, 256, 1e-5, 0, None)
    assert status == _lib.ERR_SCRATCH_LIMIT
    assert "1 MiB" in _lib.status_string(status)
