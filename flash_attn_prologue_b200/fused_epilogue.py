"""``torch.library`` custom ops of the prologue, backed by libflash_prologue.so.

Registers, under the reference's names and schemas:

* ``flash_prologue::qknorm_rope_scale_cute`` (reference:
  flash_attn_prologue/fused_epilogue.py:702-815, fake :817-828);
* ``flash_prologue::qknorm_rope_scale_cute_backward`` (reference:
  fused_epilogue.py:1304-1423, fake :1425-1437);
* the autograd link between them (reference: fused_epilogue.py:1440-1458);
* ``flash_prologue::qknorm_rope_scale_cute_inverse`` / ``_inverse_backward``
  and their autograd link (reference: fused_epilogue.py:2560-2805);
* ``flash_prologue::qknorm_rope_scale_qkv_backward``: the backward of the
  prologue on a fused [B, N, 3, H, D] QKV activation, producing its gradient
  as one tensor (no reference counterpart; the reference returns compact
  dq/dk, fused_epilogue.py:1399-1402, which autograd then gathers).

Raw-op contract kept from the reference: q/k are 4-D ``[B, H, N, D]`` views
with channel stride 1 and no expanded (stride-0) dimension, rejected with the
same ValueError texts ("expanded activations", "channel stride"); outputs and
input gradients use the compact-by-permutation strides of the inputs; sin/cos
are FP32, broadcastable to ``[B, 1, N, D/2]`` (2-D to 5-D forms accepted as in
the reference's ``_ensure_4d``). Differences by design: strided q/k/gradient
views are read in place (no clone for misalignment, no compaction copies in
backward), any ``eps > 0`` and D in {32, 64, 128, 256} with BF16/FP16/FP32 are
accepted, and the weight/scale gradients are reduced in a fixed order (no float
atomics). Nothing here runs on the CPU: the device work is the CUDA library.
"""
import ctypes
from typing import Optional, Tuple

import torch

from . import _lib

MAX_HEADS = 512
SUPPORTED_HEAD_DIMS = (32, 64, 128, 256)

_EXPANDED_MSG = "Raw CuTe does not support expanded activations; use the public frontend"
_CHANNEL_MSG = "Raw CuTe requires channel stride 1; use the public frontend"


def _get_compact_strides(shape, strides):
    """Dense strides that keep the memory order of ``strides`` (stride-0 dims stay 0).

    Same contract as the reference helper (fused_epilogue.py:688-698): dims are
    ordered by (stride, index) and packed innermost-first.
    """
    order = sorted(range(len(shape)), key=lambda i: (int(strides[i]), i))
    out = list(strides)
    running = 1
    for d in order:
        if strides[d] == 0:
            out[d] = 0
        else:
            out[d] = running
            running *= shape[d]
    return tuple(out)


def _ensure_4d(t: torch.Tensor) -> torch.Tensor:
    """sin/cos rank adaptation accepted by the reference op (fused_epilogue.py:22-32)."""
    if t.ndim == 5:
        if t.shape[2] == 1:
            return t.squeeze(2)
        if t.shape[1] == 1:
            return t.squeeze(1)
    elif t.ndim == 3:
        return t.unsqueeze(1)
    elif t.ndim == 2:
        return t.unsqueeze(0).unsqueeze(1)
    return t


def _check_raw(q: torch.Tensor, k: torch.Tensor) -> None:
    if q.numel() == 0 and k.numel() == 0:
        return  # no elements: any strides (compact strides of empty tensors hold zeros)
    if any(n > 1 and st == 0 for t in (q, k) for n, st in zip(t.shape, t.stride())):
        raise ValueError(_EXPANDED_MSG)
    if q.stride(-1) != 1 or k.stride(-1) != 1:
        raise ValueError(_CHANNEL_MSG)


def _check_common(q, k, rmsnorm_weight, scales, sin, cos, eps):
    if q.ndim != 4 or q.shape != k.shape:
        raise ValueError("q/k must be matching 4-D [B,H,N,D] tensors")
    if q.dtype not in _lib.DTYPE_CODES or k.dtype != q.dtype:
        raise ValueError("q/k must share BF16, FP16, or FP32 dtype")
    d, h = q.shape[3], q.shape[1]
    if d not in SUPPORTED_HEAD_DIMS:
        raise ValueError(f"head dimension must be one of {SUPPORTED_HEAD_DIMS}")
    if h > MAX_HEADS:
        raise ValueError(f"at most {MAX_HEADS} heads are supported")
    if not (eps > 0.0) or eps != eps or eps == float("inf"):
        raise ValueError("eps must be finite and positive")
    if tuple(rmsnorm_weight.shape) != (2, 1, d) or scales.numel() != h:
        raise ValueError("weight must be [2,1,D], log-scales must be [H,1,1]")
    # Like the reference's raw ops, which read these as Float32 whatever their
    # dtype, any floating dtype is accepted and converted to FP32 (the public
    # frontend still requires FP32, as the reference's does).
    for value in (rmsnorm_weight, scales, sin, cos):
        if not value.dtype.is_floating_point:
            raise ValueError("weights, log-scales, and sin/cos must be floating point")
    for t in (k, rmsnorm_weight, scales, sin, cos):
        if t.device != q.device:
            raise ValueError("all tensors must share a device")
    if q.device.type != "cuda":
        raise ValueError("the prologue kernels run on CUDA devices only")


def _table(t: torch.Tensor, B: int, N: int, half: int):
    """(b, n, j) element strides of a sin/cos table broadcast to [B, 1, N, D/2]."""
    t4 = _ensure_4d(t)
    if t4.dtype != torch.float32:
        t4 = t4.float()
    if t4.ndim != 4 or t4.shape[1] != 1 or t4.shape[3] != half:
        raise ValueError("sin/cos must broadcast over [B,1,N,D/2]")
    if t4.shape[0] not in (1, B) or t4.shape[2] not in (1, N):
        raise ValueError("sin/cos must broadcast over [B,1,N,D/2]")
    sb = t4.stride(0) if t4.shape[0] > 1 else 0
    sn = t4.stride(2) if t4.shape[2] > 1 else 0
    return t4, (sb, sn, t4.stride(3))


class _DeviceGuard:
    """Makes ``device`` current for the library call (which launches on it)."""

    def __init__(self, device: torch.device):
        self.index = device.index
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if self.index is not None and cur != self.index:
            self.prev = cur
            torch.cuda.set_device(self.index)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


@torch.library.custom_op("flash_prologue::qknorm_rope_scale_cute", mutates_args=())
def qknorm_rope_scale_cute_op(
    q: torch.Tensor,
    k: torch.Tensor,
    rmsnorm_weight: torch.Tensor,
    scales: torch.Tensor,
    sin: torch.Tensor,
    cos: torch.Tensor,
    eps: float = 1e-5,
) -> Tuple[torch.Tensor, torch.Tensor]:
    return cute_forward(q, k, rmsnorm_weight, scales, sin, cos, eps)


def cute_forward(q, k, rmsnorm_weight, scales, sin, cos, eps=1e-5):
    """The body of qknorm_rope_scale_cute (also called directly by the eager frontend)."""
    _check_raw(q, k)
    _check_common(q, k, rmsnorm_weight, scales, sin, cos, eps)
    B, H, N, D = (int(x) for x in q.shape)
    q_out = torch.empty_strided(q.shape, _get_compact_strides(q.shape, q.stride()),
                                dtype=q.dtype, device=q.device)
    k_out = torch.empty_strided(k.shape, _get_compact_strides(k.shape, k.stride()),
                                dtype=k.dtype, device=k.device)
    if q.numel() == 0:
        return q_out, k_out
    sin4, sin_str = _table(sin, B, N, D // 2)
    cos4, cos_str = _table(cos, B, N, D // 2)
    w = rmsnorm_weight.float().contiguous()
    s = scales.float().contiguous()
    lib = _lib.load()
    with _DeviceGuard(q.device):
        status = lib.flash_prologue_fwd(
            _lib.ptr(q), _lib.strides4(q), _lib.ptr(k), _lib.strides4(k),
            _lib.ptr(q_out), _lib.strides4(q_out), _lib.ptr(k_out), _lib.strides4(k_out),
            _lib.ptr(w), _lib.ptr(s),
            _lib.ptr(sin4), _lib.strides3(sin_str), _lib.ptr(cos4), _lib.strides3(cos_str),
            B, H, N, D, float(eps), _lib.DTYPE_CODES[q.dtype], _lib.stream_of(q.device))
    _lib.check(status, "flash_prologue_fwd")
    return q_out, k_out


@qknorm_rope_scale_cute_op.register_fake
def _qknorm_rope_scale_cute_fake(q, k, rmsnorm_weight, scales, sin, cos, eps=1e-5):
    _check_raw(q, k)
    return (
        torch.empty_strided(q.shape, _get_compact_strides(q.shape, q.stride()),
                            dtype=q.dtype, device=q.device),
        torch.empty_strided(k.shape, _get_compact_strides(k.shape, k.stride()),
                            dtype=k.dtype, device=k.device),
    )


_WORKSPACE_BYTES = {}


def bwd_workspace_bytes(B: int, H: int, N: int, D: int, dtype: torch.dtype) -> int:
    """Device workspace (bytes) of the backward launch on the current device
    (a pure function of the shape and the device, so it is queried once)."""
    import ctypes
    key = (B, H, N, D, dtype, torch.cuda.current_device())
    nbytes = _WORKSPACE_BYTES.get(key)
    if nbytes is None:
        out = ctypes.c_size_t(0)
        status = _lib.load().flash_prologue_bwd_workspace_size(B, H, N, D, _lib.DTYPE_CODES[dtype],
                                                               ctypes.byref(out))
        _lib.check(status, "flash_prologue_bwd_workspace_size")
        if len(_WORKSPACE_BYTES) >= 4096:  # many distinct shapes: start over
            _WORKSPACE_BYTES.clear()
        nbytes = _WORKSPACE_BYTES[key] = int(out.value)
    return nbytes


def _grad_view(g: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """Upstream gradient as a view the kernel reads in place (channel stride 1)."""
    if g is None:
        return torch.zeros((), dtype=like.dtype, device=like.device).expand(like.shape)
    if g.dtype != like.dtype:
        g = g.to(like.dtype)
    if g.stride(-1) != 1 and g.shape[-1] > 1:
        g = g.contiguous()
    return g


@torch.library.custom_op("flash_prologue::qknorm_rope_scale_cute_backward", mutates_args=())
def qknorm_rope_scale_cute_backward_op(
    q: torch.Tensor,
    k: torch.Tensor,
    rmsnorm_weight: torch.Tensor,
    scales: torch.Tensor,
    sin: torch.Tensor,
    cos: torch.Tensor,
    grad_q_out: torch.Tensor,
    grad_k_out: torch.Tensor,
    eps: float = 1e-5,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    return cute_backward(q, k, rmsnorm_weight, scales, sin, cos, grad_q_out, grad_k_out, eps)


def cute_backward(q, k, rmsnorm_weight, scales, sin, cos, grad_q_out, grad_k_out, eps=1e-5):
    """The body of qknorm_rope_scale_cute_backward (also called by the eager frontend)."""
    _check_raw(q, k)
    _check_common(q, k, rmsnorm_weight, scales, sin, cos, eps)
    B, H, N, D = (int(x) for x in q.shape)
    grad_q = torch.empty_strided(q.shape, _get_compact_strides(q.shape, q.stride()),
                                 dtype=q.dtype, device=q.device)
    grad_k = torch.empty_strided(k.shape, _get_compact_strides(k.shape, k.stride()),
                                 dtype=k.dtype, device=k.device)
    grad_w = torch.empty((2, 1, D), dtype=torch.float32, device=q.device)
    grad_s = torch.empty((H, 1, 1), dtype=torch.float32, device=q.device)
    gq = _grad_view(grad_q_out, q)
    gk = _grad_view(grad_k_out, k)
    sin4, sin_str = _table(sin, B, N, D // 2)
    cos4, cos_str = _table(cos, B, N, D // 2)
    w = rmsnorm_weight.float().contiguous()
    s = scales.float().contiguous()
    with _DeviceGuard(q.device):
        nbytes = bwd_workspace_bytes(B, H, N, D, q.dtype) if q.numel() else 0
        workspace = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
        _call_bwd("flash_prologue_bwd", q.device,
                  _lib.ptr(q), _lib.strides4(q), _lib.ptr(k), _lib.strides4(k),
                  _lib.ptr(w), _lib.ptr(s),
                  _lib.ptr(sin4), _lib.strides3(sin_str), _lib.ptr(cos4), _lib.strides3(cos_str),
                  _lib.ptr(gq), _lib.strides4(gq), _lib.ptr(gk), _lib.strides4(gk),
                  _lib.ptr(grad_q), _lib.strides4(grad_q), _lib.ptr(grad_k), _lib.strides4(grad_k),
                  _lib.ptr(grad_w), _lib.ptr(grad_s),
                  _lib.ptr(workspace), workspace.numel(),
                  B, H, N, D, float(eps), _lib.DTYPE_CODES[q.dtype])
    return grad_q, grad_k, grad_w, grad_s


def _call_bwd(name, device, *args):
    """Calls a backward entry point (flash_prologue_bwd / flash_prologue_inverse_bwd) on the
    device's current stream. Inside an open ``PeerGroup.reducing()`` context for the device it
    calls the entry's ``_dp`` form instead, whose finalize kernel returns d rmsnorm_weight and
    d scales already summed over the group's ranks."""
    from .distributed import active_peer_group
    lib = _lib.load()
    peers = active_peer_group(device)
    if peers is None:
        status = getattr(lib, name)(*args, _lib.stream_of(device))
    else:
        name = name + "_dp"
        status = getattr(lib, name)(*args, ctypes.byref(peers.desc), peers.next_epoch(),
                                    _lib.stream_of(device))
    _lib.check(status, name)


@qknorm_rope_scale_cute_backward_op.register_fake
def _qknorm_rope_scale_cute_backward_fake(q, k, rmsnorm_weight, scales, sin, cos, grad_q_out,
                                          grad_k_out, eps=1e-5):
    _check_raw(q, k)
    grad_q = torch.empty_strided(q.shape, _get_compact_strides(q.shape, q.stride()),
                                 dtype=q.dtype, device=q.device)
    grad_k = torch.empty_strided(k.shape, _get_compact_strides(k.shape, k.stride()),
                                 dtype=k.dtype, device=k.device)
    grad_w = torch.empty((2, 1, q.shape[-1]), device=q.device, dtype=torch.float32)
    grad_s = torch.empty((q.shape[1], 1, 1), device=q.device, dtype=torch.float32)
    return grad_q, grad_k, grad_w, grad_s


def _setup_context(ctx, inputs, output):
    q, k, rmsnorm_weight, scales, sin, cos, eps = inputs
    ctx.save_for_backward(q, k, rmsnorm_weight, scales, sin, cos)
    ctx.eps = eps


def _backward(ctx, grad_q, grad_k):
    q, k, rmsnorm_weight, scales, sin, cos = ctx.saved_tensors
    dq, dk, dw, ds = qknorm_rope_scale_cute_backward_op(
        q, k, rmsnorm_weight, scales, sin, cos, grad_q, grad_k, ctx.eps)
    return dq, dk, dw, ds, None, None, None


torch.library.register_autograd("flash_prologue::qknorm_rope_scale_cute", _backward,
                                setup_context=_setup_context)


# ---------------------------------------------------------------------------
# Inverse formulation: the forward also returns r = 1/sqrt(mean(x^2)+eps) per row,
# and the backward rebuilds the normalised rows from the outputs and r, so a
# training step need not keep q and k alive for the backward (the outputs are
# kept for attention anyway). Reference: fused_epilogue.py:2560-2805.

def _rms_shape_strides(q: torch.Tensor):
    B, H, N = (int(x) for x in q.shape[:3])
    return (B, H, N, 1), (H * N, N, 1, 1)


@torch.library.custom_op("flash_prologue::qknorm_rope_scale_cute_inverse", mutates_args=())
def qknorm_rope_scale_cute_inverse_op(
    q: torch.Tensor,
    k: torch.Tensor,
    rmsnorm_weight: torch.Tensor,
    scales: torch.Tensor,
    sin: torch.Tensor,
    cos: torch.Tensor,
    eps: float = 1e-5,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(q_out, k_out, rms_q, rms_k): the forward outputs and r per row, FP32 [B, H, N, 1]."""
    _check_raw(q, k)
    _check_common(q, k, rmsnorm_weight, scales, sin, cos, eps)
    B, H, N, D = (int(x) for x in q.shape)
    q_out = torch.empty_strided(q.shape, _get_compact_strides(q.shape, q.stride()),
                                dtype=q.dtype, device=q.device)
    k_out = torch.empty_strided(k.shape, _get_compact_strides(k.shape, k.stride()),
                                dtype=k.dtype, device=k.device)
    shape, strides = _rms_shape_strides(q)
    rms_q = torch.empty_strided(shape, strides, dtype=torch.float32, device=q.device)
    rms_k = torch.empty_strided(shape, strides, dtype=torch.float32, device=q.device)
    if q.numel() == 0:
        return q_out, k_out, rms_q, rms_k
    sin4, sin_str = _table(sin, B, N, D // 2)
    cos4, cos_str = _table(cos, B, N, D // 2)
    w = rmsnorm_weight.float().contiguous()
    s = scales.float().contiguous()
    lib = _lib.load()
    with _DeviceGuard(q.device):
        status = lib.flash_prologue_inverse_fwd(
            _lib.ptr(q), _lib.strides4(q), _lib.ptr(k), _lib.strides4(k),
            _lib.ptr(q_out), _lib.strides4(q_out), _lib.ptr(k_out), _lib.strides4(k_out),
            _lib.ptr(rms_q), _lib.ptr(rms_k), _lib.ptr(w), _lib.ptr(s),
            _lib.ptr(sin4), _lib.strides3(sin_str), _lib.ptr(cos4), _lib.strides3(cos_str),
            B, H, N, D, float(eps), _lib.DTYPE_CODES[q.dtype], _lib.stream_of(q.device))
    _lib.check(status, "flash_prologue_inverse_fwd")
    return q_out, k_out, rms_q, rms_k


@qknorm_rope_scale_cute_inverse_op.register_fake
def _qknorm_rope_scale_cute_inverse_fake(q, k, rmsnorm_weight, scales, sin, cos, eps=1e-5):
    _check_raw(q, k)
    shape, strides = _rms_shape_strides(q)
    return (
        torch.empty_strided(q.shape, _get_compact_strides(q.shape, q.stride()),
                            dtype=q.dtype, device=q.device),
        torch.empty_strided(k.shape, _get_compact_strides(k.shape, k.stride()),
                            dtype=k.dtype, device=k.device),
        torch.empty_strided(shape, strides, dtype=torch.float32, device=q.device),
        torch.empty_strided(shape, strides, dtype=torch.float32, device=q.device),
    )


def _saved_rms(rms: torch.Tensor, q_out: torch.Tensor) -> torch.Tensor:
    shape, _ = _rms_shape_strides(q_out)
    if tuple(rms.shape) != shape or rms.dtype != torch.float32 or rms.device != q_out.device:
        raise ValueError("rms_q/rms_k must be FP32 [B,H,N,1] on the activations' device")
    return rms.contiguous()


@torch.library.custom_op("flash_prologue::qknorm_rope_scale_cute_inverse_backward", mutates_args=())
def qknorm_rope_scale_cute_inverse_backward_op(
    q_out: torch.Tensor,
    k_out: torch.Tensor,
    rmsnorm_weight: torch.Tensor,
    scales: torch.Tensor,
    sin: torch.Tensor,
    cos: torch.Tensor,
    grad_q_out: torch.Tensor,
    grad_k_out: torch.Tensor,
    rms_q: torch.Tensor,
    rms_k: torch.Tensor,
    eps: float = 1e-5,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dq, dk, dw, ds) from the forward outputs and the saved r (no q/k needed)."""
    _check_raw(q_out, k_out)
    _check_common(q_out, k_out, rmsnorm_weight, scales, sin, cos, eps)
    B, H, N, D = (int(x) for x in q_out.shape)
    grad_q = torch.empty_strided(q_out.shape, _get_compact_strides(q_out.shape, q_out.stride()),
                                 dtype=q_out.dtype, device=q_out.device)
    grad_k = torch.empty_strided(k_out.shape, _get_compact_strides(k_out.shape, k_out.stride()),
                                 dtype=k_out.dtype, device=k_out.device)
    grad_w = torch.empty((2, 1, D), dtype=torch.float32, device=q_out.device)
    grad_s = torch.empty((H, 1, 1), dtype=torch.float32, device=q_out.device)
    rq = _saved_rms(rms_q, q_out)
    rk = _saved_rms(rms_k, q_out)
    gq = _grad_view(grad_q_out, q_out)
    gk = _grad_view(grad_k_out, k_out)
    sin4, sin_str = _table(sin, B, N, D // 2)
    cos4, cos_str = _table(cos, B, N, D // 2)
    w = rmsnorm_weight.float().contiguous()
    s = scales.float().contiguous()
    with _DeviceGuard(q_out.device):
        nbytes = bwd_workspace_bytes(B, H, N, D, q_out.dtype) if q_out.numel() else 0
        workspace = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q_out.device)
        _call_bwd("flash_prologue_inverse_bwd", q_out.device,
                  _lib.ptr(q_out), _lib.strides4(q_out), _lib.ptr(k_out), _lib.strides4(k_out),
                  _lib.ptr(rq), _lib.ptr(rk), _lib.ptr(w), _lib.ptr(s),
                  _lib.ptr(sin4), _lib.strides3(sin_str), _lib.ptr(cos4), _lib.strides3(cos_str),
                  _lib.ptr(gq), _lib.strides4(gq), _lib.ptr(gk), _lib.strides4(gk),
                  _lib.ptr(grad_q), _lib.strides4(grad_q), _lib.ptr(grad_k), _lib.strides4(grad_k),
                  _lib.ptr(grad_w), _lib.ptr(grad_s),
                  _lib.ptr(workspace), workspace.numel(),
                  B, H, N, D, float(eps), _lib.DTYPE_CODES[q_out.dtype])
    return grad_q, grad_k, grad_w, grad_s


@qknorm_rope_scale_cute_inverse_backward_op.register_fake
def _qknorm_rope_scale_cute_inverse_backward_fake(q_out, k_out, rmsnorm_weight, scales, sin, cos,
                                                  grad_q_out, grad_k_out, rms_q, rms_k, eps=1e-5):
    _check_raw(q_out, k_out)
    grad_q = torch.empty_strided(q_out.shape, _get_compact_strides(q_out.shape, q_out.stride()),
                                 dtype=q_out.dtype, device=q_out.device)
    grad_k = torch.empty_strided(k_out.shape, _get_compact_strides(k_out.shape, k_out.stride()),
                                 dtype=k_out.dtype, device=k_out.device)
    grad_w = torch.empty((2, 1, q_out.shape[-1]), device=q_out.device, dtype=torch.float32)
    grad_s = torch.empty((q_out.shape[1], 1, 1), device=q_out.device, dtype=torch.float32)
    return grad_q, grad_k, grad_w, grad_s


def _inverse_setup_context(ctx, inputs, output):
    q, k, rmsnorm_weight, scales, sin, cos, eps = inputs
    q_out, k_out, rms_q, rms_k = output
    ctx.save_for_backward(q_out, k_out, rmsnorm_weight, scales, sin, cos, rms_q, rms_k)
    ctx.eps = eps


def _inverse_backward(ctx, grad_q, grad_k, grad_rms_q, grad_rms_k):
    # Like the reference (fused_epilogue.py:2791-2798), gradients that reach the
    # saved statistics themselves are not propagated.
    q_out, k_out, rmsnorm_weight, scales, sin, cos, rms_q, rms_k = ctx.saved_tensors
    dq, dk, dw, ds = qknorm_rope_scale_cute_inverse_backward_op(
        q_out, k_out, rmsnorm_weight, scales, sin, cos, grad_q, grad_k, rms_q, rms_k, ctx.eps)
    return dq, dk, dw, ds, None, None, None


torch.library.register_autograd("flash_prologue::qknorm_rope_scale_cute_inverse", _inverse_backward,
                                setup_context=_inverse_setup_context)


# ---------------------------------------------------------------------------
# Backward for a fused QKV activation: one gradient tensor laid out like qkv.

def backward_into(q4, k4, rmsnorm_weight, scales, sin, cos, grad_q_out, grad_k_out, dq4, dk4,
                  eps=1e-5):
    """The prologue backward writing dq / dk into the given [B, H, N, D] views.

    dq4 / dk4 may be strided views of a larger buffer (the slots of a packed
    gradient); returns (d rmsnorm_weight [2, 1, D], d scales [H, 1, 1]).
    """
    _check_raw(q4, k4)
    _check_common(q4, k4, rmsnorm_weight, scales, sin, cos, eps)
    B, H, N, D = (int(x) for x in q4.shape)
    grad_w = torch.empty((2, 1, D), dtype=torch.float32, device=q4.device)
    grad_s = torch.empty((H, 1, 1), dtype=torch.float32, device=q4.device)
    gq = _grad_view(grad_q_out, q4)
    gk = _grad_view(grad_k_out, k4)
    sin4, sin_str = _table(sin, B, N, D // 2)
    cos4, cos_str = _table(cos, B, N, D // 2)
    w = rmsnorm_weight.float().contiguous()
    s = scales.float().contiguous()
    with _DeviceGuard(q4.device):
        nbytes = bwd_workspace_bytes(B, H, N, D, q4.dtype) if q4.numel() else 0
        workspace = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q4.device)
        _call_bwd("flash_prologue_bwd", q4.device,
                  _lib.ptr(q4), _lib.strides4(q4), _lib.ptr(k4), _lib.strides4(k4),
                  _lib.ptr(w), _lib.ptr(s),
                  _lib.ptr(sin4), _lib.strides3(sin_str), _lib.ptr(cos4), _lib.strides3(cos_str),
                  _lib.ptr(gq), _lib.strides4(gq), _lib.ptr(gk), _lib.strides4(gk),
                  _lib.ptr(dq4), _lib.strides4(dq4), _lib.ptr(dk4), _lib.strides4(dk4),
                  _lib.ptr(grad_w), _lib.ptr(grad_s),
                  _lib.ptr(workspace), workspace.numel(),
                  B, H, N, D, float(eps), _lib.DTYPE_CODES[q4.dtype])
    return grad_w, grad_s


@torch.library.custom_op("flash_prologue::qknorm_rope_scale_qkv_backward", mutates_args=())
def qknorm_rope_scale_qkv_backward_op(
    qkv: torch.Tensor,
    rmsnorm_weight: torch.Tensor,
    scales: torch.Tensor,
    sin: torch.Tensor,
    cos: torch.Tensor,
    grad_q_out: Optional[torch.Tensor],
    grad_k_out: Optional[torch.Tensor],
    grad_v: Optional[torch.Tensor],
    eps: float = 1e-5,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(grad_qkv, dw, ds) for qkv [B, N, 3, H, D].

    grad_q_out / grad_k_out are the gradients of the prologue outputs as
    [B, H, N, D] views and grad_v that of the V slot as [B, N, H, D] (None =
    zero). grad_qkv has qkv's memory order; the backward kernel writes dq and
    dk into its Q and K slots through strided output views and grad_v is
    copied into its V slot by the library's row copy, so the caller needs no
    gather of slice gradients.
    """
    if qkv.ndim != 5 or qkv.shape[2] != 3:
        raise ValueError("qkv must be [B,N,3,H,D]")
    grad_qkv = torch.empty_strided(qkv.shape, _get_compact_strides(qkv.shape, qkv.stride()),
                                   dtype=qkv.dtype, device=qkv.device)
    q4 = qkv[:, :, 0].permute(0, 2, 1, 3)
    k4 = qkv[:, :, 1].permute(0, 2, 1, 3)
    dq4 = grad_qkv[:, :, 0].permute(0, 2, 1, 3)
    dk4 = grad_qkv[:, :, 1].permute(0, 2, 1, 3)
    grad_w, grad_s = backward_into(q4, k4, rmsnorm_weight, scales, sin, cos, grad_q_out, grad_k_out,
                                   dq4, dk4, eps)
    if grad_v is None:
        grad_qkv[:, :, 2].zero_()
    else:
        _lib.copy_rows(grad_qkv[:, :, 2], grad_v)
    return grad_qkv, grad_w, grad_s


@qknorm_rope_scale_qkv_backward_op.register_fake
def _qknorm_rope_scale_qkv_backward_fake(qkv, rmsnorm_weight, scales, sin, cos, grad_q_out,
                                         grad_k_out, grad_v, eps=1e-5):
    D, H = qkv.shape[-1], qkv.shape[-2]
    return (torch.empty_strided(qkv.shape, _get_compact_strides(qkv.shape, qkv.stride()),
                                dtype=qkv.dtype, device=qkv.device),
            torch.empty((2, 1, D), dtype=torch.float32, device=qkv.device),
            torch.empty((H, 1, 1), dtype=torch.float32, device=qkv.device))
