"""Data-parallel reduction of the prologue's parameter gradients.

The prologue is per row, so tokens (packed) or batch (dense) shard across
ranks with no communication in the forward or in dq/dk. The only exchange is
the sum over ranks of the two small FP32 parameter gradients,
d rmsnorm_weight [2,1,D] and d scales [H,1,1] (2*D + H floats). The
reference has no distributed code; this is the B200 build's DP step.

Two modes over one packed [2*D + H] FP32 buffer:
* ``deterministic=True`` (default): all_gather of every rank's partial, then
  a sum in rank order on the device -- bit-identical run to run whatever the
  collective algorithm (same cost as an all-reduce at this size).
* ``deterministic=False``: one all_reduce(SUM).
"""
from typing import Iterable, Optional

import torch
import torch.distributed as dist


def pack_param_grads(dw: torch.Tensor, ds: torch.Tensor) -> torch.Tensor:
    return torch.cat((dw.reshape(-1).float(), ds.reshape(-1).float()))


def unpack_param_grads(flat: torch.Tensor, dw_like: torch.Tensor, ds_like: torch.Tensor):
    n = dw_like.numel()
    return flat[:n].view_as(dw_like), flat[n:n + ds_like.numel()].view_as(ds_like)


def reduce_param_grads(dw: torch.Tensor, ds: torch.Tensor, group: Optional[dist.ProcessGroup] = None,
                       deterministic: bool = True):
    """Returns (dw, ds) summed over the ranks of ``group`` (new tensors)."""
    flat = pack_param_grads(dw, ds)
    world = dist.get_world_size(group)
    if world == 1:
        return unpack_param_grads(flat, dw, ds)
    if deterministic:
        gathered = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
        dist.all_gather_into_tensor(gathered, flat, group=group)
        gathered = gathered.view(world, flat.numel())
        total = gathered[0].clone()
        for r in range(1, world):  # fixed rank order
            total += gathered[r]
    else:
        total = flat
        dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
    return unpack_param_grads(total, dw, ds)


def allreduce_module_grads(modules: Iterable[torch.nn.Module],
                           group: Optional[dist.ProcessGroup] = None, deterministic: bool = True):
    """Sums ``rmsnorm_weight.grad`` / ``scales.grad`` of RMSNormRoPEScale modules over ranks."""
    for m in modules:
        if m.rmsnorm_weight.grad is None or m.scales.grad is None:
            continue
        dw, ds = reduce_param_grads(m.rmsnorm_weight.grad, m.scales.grad, group, deterministic)
        m.rmsnorm_weight.grad.copy_(dw)
        m.scales.grad.copy_(ds)


def shard_range(total: int, rank: int, world: int, align: int = 1):
    """Contiguous [start, stop) of ``total`` rows for ``rank``, boundaries on ``align``."""
    units = -(-total // align)
    per = units // world
    extra = units % world
    start_u = rank * per + min(rank, extra)
    stop_u = start_u + per + (1 if rank < extra else 0)
    return min(start_u * align, total), min(stop_u * align, total)
