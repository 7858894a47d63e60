"""A library call from a thread that has made no CUDA call yet.

The TMA tensor maps are encoded with a driver call that needs a context bound
to the calling thread. A thread whose first CUDA call is into this library (an
autograd worker thread, once the workspace size is known from another thread)
has none; the library binds the device's primary context and encodes again
rather than falling back to the register path, whose parameter-gradient sums
are grouped differently. The check: flash_prologue_bwd called from a fresh
thread, on buffers the main thread allocated, gives the main thread's bits.
"""
import threading

import pytest
import torch

from flash_attn_prologue_b200 import _lib


def _bits(t):
    return t.view(torch.int16 if t.element_size() == 2 else torch.int32)


@pytest.mark.gpu
def test_backward_from_a_fresh_thread_takes_the_tma_path():
    from flash_attn_prologue_b200.fused_epilogue import bwd_workspace_bytes, _get_compact_strides
    lib = _lib.load()
    T, H, D = 2048, 16, 64
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, gq, gk = (torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(4))
    q4, k4, gq4, gk4 = (t.permute(1, 0, 2)[None] for t in (q, k, gq, gk))
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    ang = torch.rand(T, D // 2, generator=g, device="cuda") * 6
    sin, cos = ang.sin(), ang.cos()
    ws = torch.empty(bwd_workspace_bytes(1, H, T, D, q.dtype), dtype=torch.uint8, device="cuda")
    tab = _lib.strides3((0, D // 2, 1))
    stream = _lib.stream_of(q.device)

    def outputs():
        dq = torch.empty_strided(q4.shape, _get_compact_strides(q4.shape, q4.stride()), dtype=q4.dtype,
                                 device="cuda")
        return dq, torch.empty_like(dq), torch.empty(2, 1, D, device="cuda"), torch.empty(H, 1, 1, device="cuda")

    def args(o):
        dq, dk, dw, ds = o
        return (_lib.ptr(q4), _lib.strides4(q4), _lib.ptr(k4), _lib.strides4(k4), _lib.ptr(w), _lib.ptr(s),
                _lib.ptr(sin), tab, _lib.ptr(cos), tab, _lib.ptr(gq4), _lib.strides4(gq4), _lib.ptr(gk4),
                _lib.strides4(gk4), _lib.ptr(dq), _lib.strides4(dq), _lib.ptr(dk), _lib.strides4(dk),
                _lib.ptr(dw), _lib.ptr(ds), _lib.ptr(ws), ws.numel(), 1, H, T, D, 1e-5, 0, stream)

    main_out, thread_out = outputs(), outputs()
    assert lib.flash_prologue_bwd(*args(main_out)) == 0
    torch.cuda.synchronize()
    status = []
    th = threading.Thread(target=lambda: status.append(lib.flash_prologue_bwd(*args(thread_out))))
    th.start()
    th.join()
    assert status == [0]
    torch.cuda.synchronize()
    for a, b in zip(main_out, thread_out):
        assert torch.equal(_bits(a), _bits(b))
    # the register path groups the partial sums differently: it is not what ran above
    _lib.set_path(1)
    try:
        reg_out = outputs()
        assert lib.flash_prologue_bwd(*args(reg_out)) == 0
        torch.cuda.synchronize()
    finally:
        _lib.set_path(0)
    assert not torch.equal(_bits(main_out[2]), _bits(reg_out[2]))
    assert _lib.device_error(reset=True) == 0
