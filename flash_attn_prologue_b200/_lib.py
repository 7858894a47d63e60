"""ctypes binding of libflash_prologue.so (declarations: include/flash_prologue.h).

The library is built in-tree by ``python -m flash_attn_prologue_b200.build``
(or ``__graft_entry__.build()``). Loading is lazy: importing the package never
touches CUDA or the library. There is no fallback: a missing library raises.
"""
import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "libflash_prologue.so"
_lock = threading.Lock()
_lib = None

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_CHANNEL_STRIDE = 3
ERR_EXPANDED = 4
ERR_WORKSPACE = 5
ERR_CUDA = 6
ERR_ALIGNMENT = 7
ERR_SCRATCH_LIMIT = 8

DTYPE_CODES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}

_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64

SIGNATURES = {
    "flash_prologue_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "flash_prologue_version": ([], ctypes.c_int),
    "flash_prologue_fwd": ([_vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _vp,
                            _vp, _i64p, _vp, _i64p, _i64, _i64, _i64, _i64,
                            ctypes.c_float, ctypes.c_int, _vp], ctypes.c_int),
    "flash_prologue_inverse_fwd": ([_vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _vp,
                                    _vp, _vp, _vp, _i64p, _vp, _i64p, _i64, _i64, _i64, _i64,
                                    ctypes.c_float, ctypes.c_int, _vp], ctypes.c_int),
    "flash_prologue_inverse_bwd": ([_vp, _i64p, _vp, _i64p, _vp, _vp, _vp, _vp, _vp, _i64p,
                                    _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                                    _vp, _vp, _vp, ctypes.c_size_t, _i64, _i64, _i64, _i64,
                                    ctypes.c_float, ctypes.c_int, _vp], ctypes.c_int),
    "flash_prologue_bwd_workspace_size": ([_i64, _i64, _i64, _i64, ctypes.c_int,
                                           ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "flash_prologue_bwd_noalloc": ([_vp, _i64p, _vp, _i64p, _vp, _vp, _vp, _i64p, _vp, _i64p,
                                    _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _vp,
                                    _i64, _i64, _i64, _i64, ctypes.c_float, ctypes.c_int, _vp],
                                   ctypes.c_int),
    "flash_prologue_qkv_gemm_fwd": ([_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp,
                                     _vp, _i64p, _vp, _i64p, _vp, _vp, _vp, _vp, _vp,
                                     ctypes.c_float, ctypes.c_int, _vp], ctypes.c_int),
    "flash_prologue_qkv_bwd_dx": ([_vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _vp,
                                   _i64, _i64, _i64, _i64, _i64, _vp], ctypes.c_int),
    "flash_prologue_qkv_bwd_dw_workspace_size": ([_i64, _i64, _i64, _i64, _i64,
                                                  ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "flash_prologue_qkv_bwd_dw": ([_vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _vp, ctypes.c_int,
                                   _vp, ctypes.c_size_t, _i64, _i64, _i64, _i64, _i64, _vp],
                                  ctypes.c_int),
    "flash_prologue_copy_rows": ([_vp, _i64p, _vp, _i64p, _i64p, _i64, _vp], ctypes.c_int),
    "flash_prologue_set_path": ([ctypes.c_int], ctypes.c_int),
    "flash_prologue_set_gemm_variant": ([ctypes.c_int], ctypes.c_int),
    "flash_prologue_selftest_wait_timeout": ([ctypes.c_uint32, _vp], ctypes.c_int),
    "flash_prologue_device_error": ([ctypes.POINTER(ctypes.c_int), ctypes.c_int], ctypes.c_int),
    "flash_prologue_bwd": ([_vp, _i64p, _vp, _i64p, _vp, _vp, _vp, _i64p, _vp, _i64p,
                            _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _vp,
                            _vp, ctypes.c_size_t, _i64, _i64, _i64, _i64,
                            ctypes.c_float, ctypes.c_int, _vp], ctypes.c_int),
    "flash_prologue_bwd_dp": ([_vp, _i64p, _vp, _i64p, _vp, _vp, _vp, _i64p, _vp, _i64p,
                               _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _vp,
                               _vp, ctypes.c_size_t, _i64, _i64, _i64, _i64,
                               ctypes.c_float, ctypes.c_int, _vp, ctypes.c_uint32, _vp], ctypes.c_int),
    "flash_prologue_inverse_bwd_dp": ([_vp, _i64p, _vp, _i64p, _vp, _vp, _vp, _vp, _vp, _i64p,
                                       _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                                       _vp, _vp, _vp, ctypes.c_size_t, _i64, _i64, _i64, _i64,
                                       ctypes.c_float, ctypes.c_int, _vp, ctypes.c_uint32, _vp], ctypes.c_int),
    "flash_prologue_peer_buffer_bytes": ([ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(ctypes.c_size_t),
                                          ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "flash_prologue_ipc_handle": ([_vp, _vp, ctypes.POINTER(ctypes.c_int64)], ctypes.c_int),
    "flash_prologue_ipc_open": ([_vp, _i64, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "flash_prologue_ipc_close": ([_vp, _i64], ctypes.c_int),
    "flash_prologue_peer_reduce_emulated": ([_vp, _i64, ctypes.c_int32, ctypes.c_int32, _vp, _vp, _vp,
                                             ctypes.c_uint32, _vp], ctypes.c_int),
}

MAX_PEERS = 8


class PeersDesc(ctypes.Structure):
    """flash_prologue_peers (include/flash_prologue.h): every rank's exchange
    buffer and flag array as mapped in this process."""
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("max_cols", ctypes.c_int32),
                ("wait_ms", ctypes.c_int32), ("data", ctypes.c_void_p * MAX_PEERS),
                ("flags", ctypes.c_void_p * MAX_PEERS)]


class PrologueError(RuntimeError):
    """A CUDA-side failure reported by libflash_prologue.so."""


def lib_path() -> Path:
    return _LIB_PATH


def load():
    """Loads (once) and returns the ctypes handle; raises if the library is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise RuntimeError(
                    f"{_LIB_PATH.name} is not built; run `python -m flash_attn_prologue_b200.build` "
                    "(the CUDA kernels have no CPU fallback)")
            handle = ctypes.CDLL(os.fspath(_LIB_PATH))
            for name, (argtypes, restype) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = restype
            _lib = handle
    return _lib


def set_path(mode: int) -> None:
    """0: automatic (default): TMA pipeline when the layout allows, outputs by TMA
    stores where measured faster; 1: register path only; 2: TMA pipeline, outputs
    always by TMA stores; 3: TMA pipeline, outputs by the lanes' stores."""
    check(load().flash_prologue_set_path(int(mode)), "flash_prologue_set_path")


def set_gemm_variant(variant: int) -> None:
    """Fused QKV GEMM mainloop: 0 = CTA pairs (default), 1 = one CTA per SM."""
    check(load().flash_prologue_set_gemm_variant(int(variant)), "flash_prologue_set_gemm_variant")


def selftest_wait_timeout(tries: int = 4096) -> None:
    """Runs a bounded wait that times out on purpose (sets the device error word)."""
    check(load().flash_prologue_selftest_wait_timeout(int(tries), stream_of(torch.device("cuda"))),
          "flash_prologue_selftest_wait_timeout")


def device_error(reset: bool = True) -> int:
    """Device error word of the pipelined kernels (0 = none); synchronous."""
    value = ctypes.c_int(0)
    check(load().flash_prologue_device_error(ctypes.byref(value), int(reset)),
          "flash_prologue_device_error")
    return int(value.value)


def status_string(status: int) -> str:
    return load().flash_prologue_status_string(status).decode()


def check(status: int, what: str) -> None:
    """Maps a library status to the exception the reference raises for it."""
    if status == OK:
        return
    msg = f"{what}: {status_string(status)}"
    if status in (ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_CHANNEL_STRIDE, ERR_EXPANDED,
                  ERR_ALIGNMENT, ERR_WORKSPACE):
        raise ValueError(msg)
    raise PrologueError(msg)


def copy_rows(dst: torch.Tensor, src: torch.Tensor) -> None:
    """dst.copy_(src) on the device for same-shape, same-dtype tensors whose last
    dimension is contiguous, by the library's strided row copy (dimensions that
    are contiguous in both are merged into longer rows). Layouts the kernel
    cannot take (more than three outer dimensions after merging, or rows and
    strides that are not 16-byte multiples) use torch's copy."""
    if dst.shape != src.shape or dst.dtype != src.dtype:
        raise ValueError("copy_rows: shape and dtype must match")
    if dst.device.type != "cuda" or src.device != dst.device:
        raise ValueError("copy_rows: both tensors must be on the same CUDA device")
    if dst.numel() == 0:
        return
    es = dst.element_size()
    shape, ss, ds = list(dst.shape), list(src.stride()), list(dst.stride())
    # drop extent-1 dims, then merge each dim into the next when contiguous in both
    dims = [(n, a, b) for n, a, b in zip(shape, ss, ds) if n != 1] or [(1, 1, 1)]
    if dims[-1][1] != 1 or dims[-1][2] != 1:
        dst.copy_(src)
        return
    merged = [list(dims[-1])]
    for n, a, b in reversed(dims[:-1]):
        row = merged[0]
        if a == row[0] * row[1] and b == row[0] * row[2]:
            row[0] *= n
        else:
            merged.insert(0, [n, a, b])
    row_bytes = merged[-1][0] * es
    outer = merged[:-1]
    if len(outer) > 3 or row_bytes % 16:
        dst.copy_(src)
        return
    outer = [[1, 0, 0]] * (3 - len(outer)) + outer
    status = load().flash_prologue_copy_rows(
        ptr(src), strides3([o[1] * es for o in outer]), ptr(dst), strides3([o[2] * es for o in outer]),
        strides3([o[0] for o in outer]), row_bytes, stream_of(dst.device))
    if status == ERR_ALIGNMENT:
        dst.copy_(src)
        return
    check(status, "flash_prologue_copy_rows")


def strides4(t: torch.Tensor):
    return (ctypes.c_int64 * 4)(*t.stride())


def strides3(values):
    return (ctypes.c_int64 * 3)(*values)


def ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(device: torch.device):
    """The current CUDA stream of ``device`` as a cudaStream_t (a direct query
    of the raw handle where torch exposes one: a few microseconds less per call
    than building a Stream object)."""
    if _raw_stream is not None:
        index = device.index if device.index is not None else torch.cuda.current_device()
        return ctypes.c_void_p(_raw_stream(index))
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
