"""``RMSNormRoPEScale``: the prologue as an ``nn.Module`` with FP32 master parameters.

Mirrors flash_attn_prologue/layers/RMSNorm.py:141-199: constructor arguments
and checks, state-dict names/shapes (``rmsnorm_weight [2,1,D]``,
``scales [H,1,1]``), FP32 masters that survive ``.bfloat16()``/``.to()`` and
``load_state_dict(assign=True)``, ``reset_parameters`` (weight = 1,
scales = log(initial_scale), default initial_scale = D**-0.5).
"""
import math
from typing import Tuple

import torch
from torch import Tensor, nn


class RMSNormRoPEScale(nn.Module):
    """Packed/dense prologue with FP32 master affine and log-scale parameters.

    initial_scale multiplies Q only; use 1.0 when attention applies 1/sqrt(D).
    The default is 1/sqrt(D), which requires attention softmax_scale=1.
    backend="cute" runs the sm_100a CUDA kernels; "native" the PyTorch
    formulation. State-dict names/shapes: rmsnorm_weight [2,1,D], scales [H,1,1].
    """

    def __init__(self, num_heads: int, head_dim: int, eps: float = 1e-5,
                 *, initial_scale=None, backend: str = "native"):
        super().__init__()
        if num_heads <= 0 or head_dim <= 0 or head_dim % 2:
            raise ValueError("num_heads must be positive and head_dim positive/even")
        if not math.isfinite(eps) or eps <= 0:
            raise ValueError("eps must be finite and positive")
        initial_scale = head_dim ** -0.5 if initial_scale is None else initial_scale
        if not math.isfinite(initial_scale) or initial_scale <= 0:
            raise ValueError("initial_scale must be finite and positive")
        from ..functional import prepare_backend
        prepare_backend(backend)
        self.num_heads, self.head_dim, self.eps = num_heads, head_dim, eps
        self.initial_scale, self.backend = initial_scale, backend
        self.rmsnorm_weight = nn.Parameter(torch.empty(2, 1, head_dim, dtype=torch.float32))
        self.scales = nn.Parameter(torch.empty(num_heads, 1, 1, dtype=torch.float32))
        self.reset_parameters()

    def _apply(self, fn, recurse=True):
        # Device moves follow `fn`; dtype casts do not reach the FP32 masters.
        def keep_fp32(tensor):
            target = fn(tensor)
            if tensor.is_meta or target.is_meta:
                return target.float()
            return tensor.to(device=target.device, dtype=torch.float32)
        return super()._apply(keep_fp32, recurse=recurse)

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict,
                              missing_keys, unexpected_keys, error_msgs):
        # assign=True would otherwise install a lower-precision checkpoint tensor.
        for name in ("rmsnorm_weight", "scales"):
            key = prefix + name
            if key in state_dict:
                state_dict[key] = state_dict[key].float()
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict,
                                      missing_keys, unexpected_keys, error_msgs)

    def bfloat(self):
        """Alias of ``bfloat16()``; the FP32 masters stay FP32."""
        return self.bfloat16()

    def reset_parameters(self) -> None:
        nn.init.ones_(self.rmsnorm_weight)
        nn.init.constant_(self.scales, math.log(self.initial_scale))

    def forward(self, q: Tensor, k: Tensor, sin: Tensor, cos: Tensor) -> Tuple[Tensor, Tensor]:
        from ..functional import qknorm_rope_scale
        return qknorm_rope_scale(q, k, self.rmsnorm_weight, self.scales,
                                 sin, cos, self.eps, backend=self.backend)
