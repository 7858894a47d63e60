"""``FusedQKV``: QKV projection + Q/K RMSNorm + RoPE + Q scale as one module.

Mirrors flash_attn_prologue/layers/FusedQKV.py:170-205: constructor
``(hidden_size, num_heads, head_dim, eps)``, parameters ``qkv_proj.weight``
``[3*H*D, hidden]`` (nn.Linear, no bias, truncated-normal std 0.02),
``qk_norm_weight [2, 1, D]`` (ones) and ``scales [H, 1, 1]`` (log(D**-0.5)),
and ``forward(x, thetas=(sin, cos)) -> (q, k, v)`` as contiguous
``[B, H, N, D]``, raising ValueError without thetas. The reference's forward
calls an op signature its code base does not define; here the forward is the
fused tcgen05 GEMM with the prologue in its epilogue
(``flash_prologue::fused_qkv_epilogue``, given the module's eps), whose numerics are the reference's
main formulation (functional.py:89-94: FP32 math, Q scaled before the one
cast). sin/cos are the half-width tables ``[N, D/2]`` / ``[B, N, D/2]`` of
the reference's main API; full-width tables in the rotate-half convention
(both halves equal, as the reference layer's eager draft uses) are accepted
and their first half taken.
"""
import math
from typing import Optional, Tuple

import torch
from torch import Tensor, nn


class FusedQKV(nn.Module):
    def __init__(self, hidden_size: int, num_heads: int, head_dim: int, eps: float = 1e-5):
        super().__init__()
        if hidden_size <= 0 or num_heads <= 0 or head_dim <= 0 or head_dim % 2:
            raise ValueError("hidden_size, num_heads must be positive and head_dim positive/even")
        if not math.isfinite(eps) or eps <= 0:
            raise ValueError("eps must be finite and positive")
        self.hidden_size, self.num_heads, self.head_dim, self.eps = hidden_size, num_heads, head_dim, eps
        self.qkv_proj = nn.Linear(hidden_size, 3 * num_heads * head_dim, bias=False)
        self.qk_norm_weight = nn.Parameter(torch.ones(2, 1, head_dim))
        self.scales = nn.Parameter(torch.empty(num_heads, 1, 1))
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.trunc_normal_(self.qkv_proj.weight, std=0.02)
        nn.init.constant_(self.qk_norm_weight, 1.0)
        nn.init.constant_(self.scales, math.log(self.head_dim ** -0.5))

    def _half(self, t: Tensor) -> Tensor:
        return t[..., : self.head_dim // 2] if t.shape[-1] == self.head_dim else t

    def forward(self, x: Tensor, thetas: Optional[Tuple[Tensor, Tensor]] = None) -> Tuple[Tensor, Tensor, Tensor]:
        if thetas is None:
            raise ValueError("FusedQKV requires precomputed RoPE thetas (sin, cos).")
        if self.qkv_proj.weight.dtype != torch.bfloat16 or x.dtype != torch.bfloat16:
            raise ValueError("FusedQKV runs its projection in BF16: cast the module and x to torch.bfloat16")
        from ..fused_qkv import fused_qkv_epilogue_op
        sin, cos = (self._half(t).float() for t in thetas)
        q, k, v, _, _ = fused_qkv_epilogue_op(x, self.qkv_proj.weight, self.qk_norm_weight.float(),
                                              self.scales.float(), sin, cos, self.eps)
        return q, k, v

    def extra_repr(self) -> str:
        return (f"hidden_size={self.hidden_size}, num_heads={self.num_heads}, "
                f"head_dim={self.head_dim}, eps={self.eps}")
