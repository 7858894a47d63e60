"""Data-parallel reduction of the prologue's parameter gradients.

The prologue is per row, so tokens (packed) or batch (dense) shard across
ranks with no communication in the forward or in dq/dk. The only exchange is
the sum over ranks of the two small FP32 parameter gradients,
d rmsnorm_weight [2,1,D] and d scales [H,1,1] (2*D + H floats). The
reference has no distributed code; this is the B200 build's DP step.

Two modes over one packed [2*D + H] FP32 buffer:
* ``deterministic=True`` (default): all_gather of every rank's partial into a
  [world, 2*D + H] tensor, then one column sum on the device. Every rank sums
  the same gathered tensor with the same kernel, so the result is
  bit-identical on every rank and run to run whatever algorithm the collective
  uses (same cost as an all-reduce at this size). Three launches: pack,
  all_gather, sum.
* ``deterministic=False``: one all_reduce(SUM).

``ParamGradReducer`` issues the reduction on a side stream once the backward
has produced the partials, so it overlaps whatever the main stream runs next
(the next step's forward, or the rest of a model's backward); ``wait()`` joins
the results back into the main stream before they are used.
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
        total = gathered.view(world, flat.numel()).sum(0)
    else:
        total = flat
        dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
    return unpack_param_grads(total, dw, ds)


class ParamGradReducer:
    """reduce_param_grads on a side stream, overlapping the main stream's next work.

    ``reduce(dw, ds)`` orders the side stream after the work the current
    stream has queued (the backward that produced dw, ds), issues the
    reduction there and returns its (dw, ds) results; ``wait()`` makes the
    current stream wait for every reduction issued so far. Use the results
    only after ``wait()``. Every rank must call ``reduce`` the same number of
    times in the same order (it issues a collective).
    """

    def __init__(self, group: Optional[dist.ProcessGroup] = None, deterministic: bool = True,
                 device: Optional[torch.device] = None):
        self.group = group
        self.deterministic = deterministic
        self.stream = torch.cuda.Stream(device) if torch.cuda.is_available() else None

    def reduce(self, dw: torch.Tensor, ds: torch.Tensor):
        if self.stream is None or not dw.is_cuda:
            return reduce_param_grads(dw, ds, self.group, self.deterministic)
        main = torch.cuda.current_stream(dw.device)
        self.stream.wait_stream(main)
        with torch.cuda.stream(self.stream):
            out = reduce_param_grads(dw, ds, self.group, self.deterministic)
        # The partials were allocated on the main stream and are read here; the
        # results, allocated here, are read on the main stream after wait().
        dw.record_stream(self.stream)
        ds.record_stream(self.stream)
        for t in out:
            t.record_stream(main)
        return out

    def wait(self):
        if self.stream is not None:
            torch.cuda.current_stream(self.stream.device).wait_stream(self.stream)


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
