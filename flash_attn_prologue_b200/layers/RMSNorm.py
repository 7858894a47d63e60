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


_MASTERS = ("rmsnorm_weight", "scales")


def _keep_fp32_dtype(fn):
    """Wraps a Module._apply conversion so that it never changes a tensor's dtype.

    The conversion is first tried on an empty tensor of the same dtype and
    device. If that keeps the dtype (a device move, ``share_memory_``,
    ``to_empty``), the conversion itself runs. If it changes the dtype
    (``.bfloat16()``, ``.half()``, ``.to(dtype)``, with or without a device
    move), the tensor goes to the probe's device and stays FP32, so its values
    are never rounded through the narrower type.
    """
    def convert(t):
        probe = fn(t.new_empty(0))
        if probe.dtype == t.dtype:
            return fn(t)
        if t.is_meta:
            return fn(t).float()
        return t.to(device=probe.device, dtype=torch.float32)
    return convert


def _masters_back_to_fp32(module, incompatible_keys):
    """load_state_dict(..., assign=True) installs the checkpoint's own tensors;
    a lower-precision one is widened back to an FP32 parameter (exactly)."""
    for name in _MASTERS:
        p = module._parameters.get(name)
        if p is not None and p.dtype != torch.float32:
            module._parameters[name] = nn.Parameter(p.detach().float(), requires_grad=p.requires_grad)


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
        self.register_load_state_dict_post_hook(_masters_back_to_fp32)

    def _apply(self, fn, recurse=True):
        return super()._apply(_keep_fp32_dtype(fn), recurse=recurse)

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
