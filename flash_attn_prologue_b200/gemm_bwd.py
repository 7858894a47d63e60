"""The projection backward under the reference's module path (flash_attn_prologue/gemm_bwd.py).

``matmul_bwd_dx``, ``matmul_bwd_dw`` and ``fused_qkv_backward`` (and their
``torch.ops.flash_prologue`` ops) are defined in ``fused_qkv`` next to the
forward ops they differentiate; they run the tcgen05 backward GEMM kernels
that read the per-head gradients in place.
"""
from .fused_qkv import fused_qkv_backward, matmul_bwd_dw, matmul_bwd_dx  # noqa: F401

__all__ = ["matmul_bwd_dx", "matmul_bwd_dw", "fused_qkv_backward"]
