"""The allocation-free backward entry point, flash_prologue_bwd_noalloc.

It serves callers that cannot allocate device memory per call (runtimes that
plan all device memory up front, host-language bindings without a device
allocator); its scratch is a static 1 MiB array inside the library. Checked
here through the C ABI against the existing entry point (flash_prologue_bwd,
reached through the flash_prologue::qknorm_rope_scale_cute_backward op): both
run the same kernels on the same grid, so every result must be bit-identical.
Each kernel path (TMA pipeline and register path) runs a sequence of calls in a
row with different inputs and grid sizes -- a large grid, then a small one, then
the large one again -- so partial rows a previous call left in the shared
scratch are present and must not leak into the next result; and a problem too
large for the scratch is rejected. This file is collected last, so a run that
stops at the first failure has run every other test before it.
"""
import ctypes

import pytest
import torch

from flash_attn_prologue_b200 import _lib, prepare_backend
from flash_attn_prologue_b200.fused_epilogue import _get_compact_strides

pytestmark = pytest.mark.gpu

# (T, H, D, packed): packed [T, H, D] views of a fused QKV buffer (heads inner),
# or dense [1, H, T, D] tensors (positions inner). The first needs the full
# persistent grid, the second a few dozen CTAs.
SEQUENCE = [(4096, 8, 64, True), (300, 4, 128, True), (4096, 8, 64, True), (700, 2, 128, False)]


def _problem(seed, T, H, D, packed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    if packed:
        buf = torch.randn(T, 3, H, D, generator=g, device="cuda").to(torch.bfloat16)
        q4 = buf[:, 0].permute(1, 0, 2)[None]
        k4 = buf[:, 1].permute(1, 0, 2)[None]
    else:
        q4, k4 = (torch.randn(1, H, T, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(2))
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    ang = torch.randn(T, D // 2, generator=g, device="cuda")
    sin, cos = ang.sin(), ang.cos()
    gq4, gk4 = (torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16).permute(1, 0, 2)[None]
                for _ in range(2))
    return q4, k4, w, s, sin, cos, gq4, gk4


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


@pytest.mark.parametrize("path", [0, 1], ids=["tma", "register"])
def test_noalloc_backward_equals_workspace_backward(path):
    prepare_backend("cute")
    try:
        _lib.set_path(path)
        for i, shape in enumerate(SEQUENCE):  # calls in a row: different inputs and grids
            args = _problem(10 * path + i, *shape)
            got = _call_noalloc(*args)
            ref = _call_existing(*args)
            torch.cuda.synchronize()
            for a, b, nm in zip(got, ref, ("dq", "dk", "drmsnorm_weight", "dscales")):
                assert a.shape == b.shape and torch.equal(a, b), (shape, nm)
    finally:
        _lib.set_path(0)
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
