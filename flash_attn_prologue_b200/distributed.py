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

``PeerGroup`` replaces the library collective altogether: inside its
``reducing()`` context the backward's own finalize kernel exchanges the
parameter-gradient sums with the other ranks over NVLink peer memory.
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


class PeerGroup:
    """The ranks' exchange buffers mapped into every rank, for flash_prologue_bwd_dp.

    Collective to build (every rank of ``group`` calls it): each rank allocates
    one small exchange buffer and flag array (zeros, from torch's allocator),
    exports IPC handles for them, gathers every rank's handles over the process
    group and maps the peers' buffers. Inside ``with group.reducing():`` every
    prologue backward on this device (qknorm_rope_scale(backend="cute"), its
    inverse form, qknorm_rope_scale_qkv and the fused QKV projection's backward)
    returns d rmsnorm_weight and d scales already summed over the ranks: its finalize
    kernel adds the per-CTA partials, exchanges the [2*D + H] sums over NVLink
    and adds them in rank order (identical bits on every rank) -- no separate
    collective, no NCCL. ``max_cols`` bounds 2*D + H (rounded up to 32).
    All ranks must run the same backward calls in the same order inside the
    context. One process per GPU on one node, at most 8 ranks (two ranks on
    one GPU are refused: their kernels would wait on each other). A rank that
    does not arrive within ``wait_ms`` leaves NaN gradients and the device
    error word set on the others instead of a hang.
    """

    def __init__(self, group: Optional[dist.ProcessGroup] = None, max_cols: int = 1024,
                 device: Optional[torch.device] = None, wait_ms: int = 2000):
        import ctypes
        from . import _lib
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.MAX_PEERS:
            raise ValueError(f"PeerGroup spans at most {_lib.MAX_PEERS} ranks")
        if not 0 < wait_ms <= 60000:
            raise ValueError("wait_ms must be in 1 .. 60000")
        self.max_cols = -(-max_cols // 32) * 32
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        nd, nf = ctypes.c_size_t(), ctypes.c_size_t()
        _lib.check(lib.flash_prologue_peer_buffer_bytes(self.world, self.max_cols, ctypes.byref(nd),
                                                        ctypes.byref(nf)), "flash_prologue_peer_buffer_bytes")
        self.data = torch.zeros(nd.value // 4, dtype=torch.float32, device=self.device)
        self.flags = torch.zeros(nf.value // 4, dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        mine = [str(torch.cuda.get_device_properties(self.device).uuid)]
        for t in (self.data, self.flags):
            h = (ctypes.c_char * 64)()
            off = ctypes.c_int64()
            _lib.check(lib.flash_prologue_ipc_handle(_lib.ptr(t), h, ctypes.byref(off)), "flash_prologue_ipc_handle")
            mine.append((bytes(h), off.value))
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=group)
        if len({e[0] for e in every}) != self.world:
            raise ValueError("PeerGroup needs one GPU per rank")
        self._opened = []
        self.desc = _lib.PeersDesc()
        self.desc.world, self.desc.rank, self.desc.max_cols = self.world, self.rank, self.max_cols
        self.desc.wait_ms = wait_ms
        for r, (_, (hd, od), (hf, of)) in enumerate(every):
            if r == self.rank:
                pd, pf = self.data.data_ptr(), self.flags.data_ptr()
            else:
                pd, pf = (self._open(lib, h, o) for h, o in ((hd, od), (hf, of)))
            self.desc.data[r], self.desc.flags[r] = pd, pf
        self.epoch = 0
        dist.barrier(group=group)

    def _open(self, lib, handle, offset):
        import ctypes
        from . import _lib
        p = ctypes.c_void_p()
        _lib.check(lib.flash_prologue_ipc_open(handle, offset, ctypes.byref(p)), "flash_prologue_ipc_open")
        self._opened.append((p.value, offset))
        return p.value

    def next_epoch(self) -> int:
        self.epoch += 1
        return self.epoch

    def reducing(self):
        """Context in which this device's cute backward reduces over the group."""
        import contextlib

        @contextlib.contextmanager
        def ctx():
            prev = _ACTIVE_PEER_GROUPS.get(self.device.index)
            _ACTIVE_PEER_GROUPS[self.device.index] = self
            try:
                yield self
            finally:
                if prev is None:
                    _ACTIVE_PEER_GROUPS.pop(self.device.index, None)
                else:
                    _ACTIVE_PEER_GROUPS[self.device.index] = prev
        return ctx()

    def close(self):
        """Unmaps the peers' buffers (after every rank's last use: call it after a barrier)."""
        from . import _lib
        lib = _lib.load()
        torch.cuda.synchronize(self.device)
        for p, off in self._opened:
            lib.flash_prologue_ipc_close(p, off)
        self._opened = []


_ACTIVE_PEER_GROUPS = {}


def active_peer_group(device: torch.device):
    """The PeerGroup whose reducing() context is open for ``device``, or None."""
    return _ACTIVE_PEER_GROUPS.get(device.index) if _ACTIVE_PEER_GROUPS else None


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
