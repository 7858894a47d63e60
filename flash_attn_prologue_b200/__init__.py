"""B200-native (sm_100a) attention prologue: Q/K RMSNorm -> split-half RoPE -> Q scale.

Public API (same names as flash_attn_prologue/__init__.py:1-19):
``qknorm_rope_scale``, ``prepare_backend``, ``RMSNormRoPEScale``. The custom-op
callables are exported lazily under the reference's names, so importing the
package touches neither CUDA nor the shared library, and changes no
environment variable.
"""
from importlib import import_module

from .functional import prepare_backend, qknorm_rope_scale, qknorm_rope_scale_qkv
from .layers.FusedQKV import FusedQKV
from .layers.RMSNorm import RMSNormRoPEScale

__version__ = "0.2.0"

_LAZY = {
    "qknorm_rope_scale_op": ("epilogue_kernel", "qknorm_rope_scale_op"),
    "qknorm_rope_scale_cute_op": ("fused_epilogue", "qknorm_rope_scale_cute_op"),
    "qknorm_rope_scale_cute_backward_op": ("fused_epilogue", "qknorm_rope_scale_cute_backward_op"),
    "qknorm_rope_scale_cute_inverse_op": ("fused_epilogue", "qknorm_rope_scale_cute_inverse_op"),
    "qknorm_rope_scale_cute_inverse_backward_op": ("fused_epilogue",
                                                   "qknorm_rope_scale_cute_inverse_backward_op"),
    "fused_qkv": ("fused_qkv", "fused_qkv_op"),
    "fused_qkv_epilogue": ("fused_qkv", "fused_qkv_epilogue_op"),
    "fused_qkv_epilogue_ckp": ("fused_qkv", "fused_qkv_epilogue_ckp_op"),
    "matmul_bwd_dx": ("gemm_bwd", "matmul_bwd_dx"),
    "matmul_bwd_dw": ("gemm_bwd", "matmul_bwd_dw"),
    "fused_qkv_backward": ("gemm_bwd", "fused_qkv_backward"),
}
__all__ = ["qknorm_rope_scale", "qknorm_rope_scale_qkv", "prepare_backend", "RMSNormRoPEScale", "FusedQKV",
           *_LAZY]


def __getattr__(name):
    if name not in _LAZY:
        raise AttributeError(name)
    module, symbol = _LAZY[name]
    import_module(f".{module}", __name__)
    # Importing a submodule binds the package attribute of the same name to
    # the module (``fused_qkv`` collides with the op alias), also for the
    # submodules it imports in turn: restore every alias whose source module
    # is loaded by now.
    import sys
    for alias, (source, exported) in _LAZY.items():
        mod = sys.modules.get(f"{__name__}.{source}")
        if mod is not None:
            globals()[alias] = getattr(mod, exported)
    return globals()[name]
