"""The C-ABI library: loads without a GPU, exports every declared entry point,
and rejects bad arguments before touching the device (CPU-only)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from flash_attn_prologue_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        text = header.read_text()
        names += re.findall(r"FLASH_PROLOGUE_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 5, names
    for name in names:
        assert hasattr(lib, name), name


def test_every_declared_symbol_has_a_python_signature():
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.flash_prologue_version() >= 100
    assert _lib.status_string(0) == "ok"
    assert "channel stride" in _lib.status_string(_lib.ERR_CHANNEL_STRIDE)
    assert "expanded activations" in _lib.status_string(_lib.ERR_EXPANDED)
    assert _lib.status_string(999) == "unknown status"


def _fwd(q_str=(0, 64, 1024, 1), D=64, eps=1e-5, dtype=0, B=1, H=16, N=4, null=False):
    lib = _lib.load()
    p = None if null else ctypes.c_void_p(16)  # never dereferenced: rejected first
    s4 = (ctypes.c_int64 * 4)(*q_str)
    o4 = (ctypes.c_int64 * 4)(0, 64, 1024, 1)
    t3 = (ctypes.c_int64 * 3)(0, 32, 1)
    return lib.flash_prologue_fwd(p, s4, p, s4, p, o4, p, o4, p, p, p, t3, p, t3,
                                  B, H, N, D, eps, dtype, None)


@pytest.mark.parametrize("kwargs,status", [
    (dict(D=48), _lib.ERR_UNSUPPORTED),
    (dict(D=512), _lib.ERR_UNSUPPORTED),
    (dict(dtype=7), _lib.ERR_UNSUPPORTED),
    (dict(H=513), _lib.ERR_UNSUPPORTED),
    (dict(eps=0.0), _lib.ERR_INVALID_ARGUMENT),
    (dict(eps=float("nan")), _lib.ERR_INVALID_ARGUMENT),
    (dict(eps=float("inf")), _lib.ERR_INVALID_ARGUMENT),
    (dict(B=-1), _lib.ERR_INVALID_ARGUMENT),
    (dict(q_str=(0, 64, 1024, 2)), _lib.ERR_CHANNEL_STRIDE),
    (dict(q_str=(0, 0, 1024, 1)), _lib.ERR_EXPANDED),
    (dict(null=True), _lib.ERR_INVALID_ARGUMENT),
    (dict(N=0, null=True), _lib.OK),  # empty problem: no launch, no device access
])
def test_fwd_argument_checks(kwargs, status):
    assert _fwd(**kwargs) == status


def test_path_modes_accepted_and_rejected():
    """Modes 0-3 (automatic, register path, TMA-stored outputs, lane-stored
    outputs) are accepted; anything else is an invalid argument and leaves the
    current mode unchanged."""
    lib = _lib.load()
    try:
        for mode in (1, 2, 3, 0):
            assert lib.flash_prologue_set_path(mode) == 0
        for mode in (-1, 4, 99):
            assert lib.flash_prologue_set_path(mode) == 1  # FLASH_PROLOGUE_ERR_INVALID_ARGUMENT
        with pytest.raises(Exception):
            _lib.set_path(4)
    finally:
        lib.flash_prologue_set_path(0)


def test_bwd_workspace_size_argument_checks():
    lib = _lib.load()
    n = ctypes.c_size_t(123)
    assert lib.flash_prologue_bwd_workspace_size(1, 16, 0, 64, 0, ctypes.byref(n)) == _lib.OK
    assert n.value == 0
    assert lib.flash_prologue_bwd_workspace_size(1, 16, 8, 40, 0, ctypes.byref(n)) == _lib.ERR_UNSUPPORTED
    assert lib.flash_prologue_bwd_workspace_size(1, 16, 8, 64, 0, None) == _lib.ERR_INVALID_ARGUMENT


def _bwd_dx(B=1, H=4, N=8, D=64, hidden=128, w=16, out=16, null_strides=False):
    lib = _lib.load()
    g = ctypes.c_void_p(16)  # never dereferenced: rejected first
    s4 = None if null_strides else (ctypes.c_int64 * 4)(H * N * D, N * D, D, 1)
    return lib.flash_prologue_qkv_bwd_dx(g, s4, g, s4, g, s4, w and ctypes.c_void_p(w),
                                         out and ctypes.c_void_p(out), B, H, N, D, hidden, None)


@pytest.mark.parametrize("kwargs,status", [
    (dict(D=32), _lib.ERR_UNSUPPORTED),
    (dict(H=3), _lib.ERR_UNSUPPORTED),            # H * D not a multiple of 256
    (dict(hidden=100), _lib.ERR_UNSUPPORTED),
    (dict(B=-1), _lib.ERR_INVALID_ARGUMENT),
    (dict(w=0), _lib.ERR_INVALID_ARGUMENT),
    (dict(null_strides=True), _lib.ERR_INVALID_ARGUMENT),
    (dict(w=24), _lib.ERR_ALIGNMENT),
    (dict(N=0, w=0, out=0), _lib.OK),             # empty sum over no tokens: nothing to write
])
def test_projection_backward_argument_checks(kwargs, status):
    assert _bwd_dx(**kwargs) == status


def test_projection_backward_dw_workspace_and_empty_accumulate():
    lib = _lib.load()
    n = ctypes.c_size_t(123)
    assert lib.flash_prologue_qkv_bwd_dw_workspace_size(2, 4, 0, 64, 128, ctypes.byref(n)) == _lib.OK
    assert n.value == 0
    assert lib.flash_prologue_qkv_bwd_dw_workspace_size(2, 4, 8, 32, 128, ctypes.byref(n)) == _lib.ERR_UNSUPPORTED
    assert lib.flash_prologue_qkv_bwd_dw_workspace_size(2, 4, 8, 64, 128, None) == _lib.ERR_INVALID_ARGUMENT
    s4 = (ctypes.c_int64 * 4)(0, 0, 64, 1)
    p = ctypes.c_void_p(16)
    # accumulate into grad_w over zero tokens: leaves it as it is, touches nothing
    assert lib.flash_prologue_qkv_bwd_dw(p, s4, p, s4, p, s4, p, p, 1, None, 0,
                                         2, 4, 0, 64, 128, None) == _lib.OK


def test_check_maps_status_to_reference_exceptions():
    with pytest.raises(ValueError, match="channel stride"):
        _lib.check(_lib.ERR_CHANNEL_STRIDE, "x")
    with pytest.raises(ValueError, match="expanded activations"):
        _lib.check(_lib.ERR_EXPANDED, "x")
    with pytest.raises(_lib.PrologueError):
        _lib.check(_lib.ERR_CUDA, "x")


def test_ops_register_and_fake_shapes_on_meta():
    """Schemas, fake impls and compact output strides, without a device."""
    from flash_attn_prologue_b200 import fused_epilogue  # noqa: F401
    q = torch.empty_strided((1, 16, 8, 64), (64 * 3 * 16 * 8, 64, 3 * 16 * 64, 1), device="meta",
                            dtype=torch.bfloat16)
    w = torch.empty(2, 1, 64, device="meta")
    s = torch.empty(16, 1, 1, device="meta")
    t = torch.empty(1, 1, 8, 32, device="meta")
    qo, ko = torch.ops.flash_prologue.qknorm_rope_scale_cute(q, q, w, s, t, t, 1e-5)
    assert qo.shape == q.shape and qo.stride() == (16 * 8 * 64, 64, 16 * 64, 1)
    dq, dk, dw, ds = torch.ops.flash_prologue.qknorm_rope_scale_cute_backward(q, q, w, s, t, t, qo, ko, 1e-5)
    assert dq.stride() == qo.stride() and dw.shape == (2, 1, 64) and ds.shape == (16, 1, 1)
    with pytest.raises(ValueError, match="expanded activations"):
        expanded = torch.empty(1, 1, 8, 64, device="meta", dtype=torch.bfloat16).expand(1, 16, 8, 64)
        torch.ops.flash_prologue.qknorm_rope_scale_cute(expanded, q, w, s, t, t, 1e-5)


def test_compact_strides_match_reference_contract():
    from flash_attn_prologue_b200.fused_epilogue import _get_compact_strides
    # packed [T,H,D] view of a [T,3,H,D] buffer -> contiguous [T,H,D] order
    assert _get_compact_strides((1, 16, 100, 64), (0, 64, 3072, 1)) == (0, 64, 1024, 1)
    assert _get_compact_strides((1, 16, 100, 64), (1, 64, 3072, 1)) == (1, 64, 1024, 1)
    assert _get_compact_strides((2, 4, 17, 32), (2176, 544, 32, 1)) == (2176, 544, 32, 1)
    assert _get_compact_strides((2, 4, 17, 32), (2176, 1, 128, 4)) == (2176, 1, 128, 4)


def test_lazy_exports_resolve_to_ops_in_any_order():
    """Package aliases under the reference's names stay the ops whichever submodule loads first
    (``fused_qkv`` is also a submodule name); gemm_bwd keeps the reference's module path."""
    import subprocess
    import sys
    # Importing the submodule directly binds the package attribute to the
    # module, as in the reference; the next lazy lookup restores every alias.
    # The package stays a plain module object (torch.compile imports it).
    first = (
        "import types\n"
        "import flash_attn_prologue_b200 as f\n"
        "assert type(f) is types.ModuleType\n"
        "import flash_attn_prologue_b200.fused_qkv\n"
        "e = f.fused_qkv_epilogue\n"
        "from flash_attn_prologue_b200.fused_qkv import fused_qkv_op\n"
        "assert f.fused_qkv is fused_qkv_op, repr(f.fused_qkv)\n"
    )
    subprocess.run([sys.executable, "-c", first], check=True, cwd=ROOT)
    code = (
        "import flash_attn_prologue_b200 as f\n"
        "a = f.matmul_bwd_dx\n"
        "assert 'CustomOpDef' in repr(f.fused_qkv), repr(f.fused_qkv)\n"
        "assert 'CustomOpDef' in repr(f.fused_qkv_epilogue)\n"
        "from flash_attn_prologue_b200.gemm_bwd import fused_qkv_backward, matmul_bwd_dw\n"
        "assert f.fused_qkv_backward is fused_qkv_backward\n"
    )
    subprocess.run([sys.executable, "-c", code], check=True, cwd=ROOT)
