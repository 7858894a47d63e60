"""Loader of the reference-generated golden vectors (see make_golden.py)."""
import json
from pathlib import Path

import numpy as np
import torch

PATH = Path(__file__).resolve().parent / "prologue_golden.npz"
DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}


def _tensor(arr: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    if dtype == torch.float32:
        return torch.from_numpy(np.array(arr, dtype=np.float32))
    return torch.from_numpy(np.array(arr, dtype=np.uint16).view(np.int16)).view(dtype)


class GoldenCase:
    """One reference case: inputs, reference outputs and gradients as CPU tensors."""

    def __init__(self, name, meta, arrays):
        self.name = name
        self.meta = meta
        self.dtype = DTYPES[meta["dtype"]]
        self.eps = meta["eps"]
        act = ("q", "k", "gq", "gk", "q_out", "k_out", "dq", "dk")
        for key in ("q", "k", "w", "s", "sin", "cos", "gq", "gk", "q_out", "k_out", "dq", "dk",
                    "dw", "ds"):
            arr = arrays[f"{name}/{key}"]
            setattr(self, key, _tensor(arr, self.dtype) if key in act else
                    torch.from_numpy(np.array(arr, dtype=np.float32)))

    @property
    def packed(self):
        return self.q.ndim == 3

    def args(self, device="cpu"):
        """(q, k, w, s, sin, cos) on ``device`` with the case's view layout."""
        q, k = self.q.to(device), self.k.to(device)
        if self.meta.get("noncontig"):
            q, k = (_interleaved(t) for t in (q, k))
        elif self.meta["layout"] == "qkv_packed":
            t, h, d = q.shape
            buf = torch.zeros((t, 3, h, d), dtype=q.dtype, device=device)
            buf[:, 0], buf[:, 1] = q, k
            q, k = buf[:, 0], buf[:, 1]
        return (q, k, self.w.to(device), self.s.to(device), self.sin.to(device),
                self.cos.to(device))


def _interleaved(x: torch.Tensor) -> torch.Tensor:
    """x as a channel-stride-2 view (the reference tests' `[..., ::2]` layout)."""
    buf = torch.zeros((*x.shape[:-1], 2 * x.shape[-1]), dtype=x.dtype, device=x.device)
    buf[..., ::2] = x
    return buf[..., ::2]


def load_golden():
    data = np.load(PATH)
    meta = json.loads(bytes(data["__meta__"]).decode())
    arrays = {k: data[k] for k in data.files if k != "__meta__"}
    return {name: GoldenCase(name, m, arrays) for name, m in sorted(meta.items())}
