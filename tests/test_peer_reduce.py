"""Data-parallel reduction of the parameter gradients over peer memory.

flash_prologue_bwd_dp's finalize kernel adds the backward's per-CTA partials
and exchanges the [2*D + H] sums with the other ranks through their mapped
exchange buffers. GPU, on one device:

* the protocol itself, every rank emulated by one cooperative launch
  (flash_prologue_peer_reduce_emulated): 1, 2, 3 and 8 ranks, three calls in
  a row (both halves of the buffers, then the first again), every rank's
  result bit-identical to the fixed-order sum restated in numpy (warp-strided
  partial rows, warps in order, ranks in order);
* flash_prologue_bwd_dp with a one-rank group gives flash_prologue_bwd's bits;
* PeerGroup in a one-rank NCCL process group: inside ``reducing()`` each
  backward path (regular, inverse, packed QKV gradient) goes through its _dp
  entry and equals the plain call bit for bit; the IPC export works;
* a rank that never arrives: the wait gives up after the descriptor's
  wait_ms, the gradients come out NaN, the device error word is set, and the
  context stays usable (one kernel, no second launch waited on);
* one process per visible GPU (2 to 8 GPUs): every rank holds the rank-order
  sum of the ranks' own gradients, bit for bit.

CPU: argument checks that return before touching the device, and PeerGroup's
own checks on a one-rank gloo group.
"""
import ctypes
import datetime
import os
import socket

import numpy as np
import pytest
import torch

from flash_attn_prologue_b200 import _lib


def _finalize_order(partials):
    """[G, C] float32 -> [C]: the finalize kernel's order (8 warps over rows w, w+8, ...)."""
    G, C = partials.shape
    out = np.zeros(C, dtype=np.float32)
    for c in range(C):
        warp_sums = []
        for w in range(8):
            v = np.float32(0)
            for g in range(w, G, 8):
                v = np.float32(v + partials[g, c])
            warp_sums.append(v)
        s = np.float32(0)
        for v in warp_sums:
            s = np.float32(s + v)
        out[c] = s
    return out


def _bits(t):
    return t.view(torch.int16 if t.element_size() == 2 else torch.int32)


def _desc(world, rank, max_cols, datas, flags):
    d = _lib.PeersDesc()
    d.world, d.rank, d.max_cols = world, rank, max_cols
    for r in range(world):
        d.data[r] = datas[r].data_ptr()
        d.flags[r] = flags[r].data_ptr()
    return d


def _buffers(world, max_cols, device):
    nd, nf = ctypes.c_size_t(), ctypes.c_size_t()
    assert _lib.load().flash_prologue_peer_buffer_bytes(world, max_cols, ctypes.byref(nd), ctypes.byref(nf)) == 0
    datas = [torch.zeros(nd.value // 4, dtype=torch.float32, device=device) for _ in range(world)]
    flags = [torch.zeros(nf.value // 4, dtype=torch.int32, device=device) for _ in range(world)]
    return datas, flags


def test_argument_checks_without_a_device_call():
    lib = _lib.load()
    nd, nf = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.flash_prologue_peer_buffer_bytes(4, 160, ctypes.byref(nd), ctypes.byref(nf)) == 0
    assert (nd.value, nf.value) == (2 * 4 * 160 * 4, 2 * 4 * 5 * 4)
    assert lib.flash_prologue_peer_buffer_bytes(9, 160, ctypes.byref(nd), ctypes.byref(nf)) == _lib.ERR_INVALID_ARGUMENT
    assert lib.flash_prologue_peer_buffer_bytes(2, 100, ctypes.byref(nd), ctypes.byref(nf)) == _lib.ERR_INVALID_ARGUMENT
    null = ctypes.c_void_p(0)
    assert lib.flash_prologue_peer_reduce_emulated(null, 1, 32, 16, null, null, null, 1, None) == \
        _lib.ERR_INVALID_ARGUMENT
    s4 = _lib.strides4(torch.empty(1, 1, 1, 1))
    t3 = _lib.strides3((0, 32, 1))
    # no group, epoch 0, a rank outside the group, a row too short for 2*D + H
    for desc, epoch in ((None, 1), (_desc_bad(rank=0, world=1, max_cols=160), 0),
                        (_desc_bad(rank=2, world=2, max_cols=160), 1), (_desc_bad(rank=0, world=1, max_cols=64), 1)):
        st = lib.flash_prologue_bwd_dp(null, s4, null, s4, null, null, null, t3, null, t3, null, s4, null, s4,
                                       null, s4, null, s4, null, null, null, 0, 1, 16, 8, 64, 1e-5, 0,
                                       ctypes.byref(desc) if desc is not None else None, epoch, None)
        assert st == _lib.ERR_INVALID_ARGUMENT


def test_peer_group_rejects_bad_arguments_before_any_device_work():
    """PeerGroup's host checks run first: a one-rank gloo group on CPU reaches them."""
    import torch.distributed as dist
    from flash_attn_prologue_b200.distributed import PeerGroup
    started = False
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ["MASTER_PORT"] = str(_free_port())
        dist.init_process_group("gloo", rank=0, world_size=1, timeout=datetime.timedelta(seconds=30))
        started = True
    try:
        for bad in (0, -5, 60001):
            with pytest.raises(ValueError, match="wait_ms"):
                PeerGroup(wait_ms=bad)
    finally:
        if started:
            dist.destroy_process_group()


def _desc_bad(rank, world, max_cols):
    d = _lib.PeersDesc()
    d.world, d.rank, d.max_cols = world, rank, max_cols
    for r in range(world):
        d.data[r] = 16
        d.flags[r] = 16
    return d


@pytest.mark.gpu
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_emulated_group_reduction_bits(world):
    """Every emulated rank gets the rank-order sum of the ranks' fixed-order sums, bit for bit."""
    lib = _lib.load()
    G, D, H = 37, 64, 16
    C, two_d, max_cols = 2 * D + H, 2 * D, 160
    datas, flags = _buffers(world, max_cols, "cuda")
    desc = _desc(world, 0, max_cols, datas, flags)
    rng = np.random.default_rng(world)
    for epoch in (1, 2, 3):  # both halves of the buffers, then the first again
        parts = [rng.standard_normal((G, C), dtype=np.float32) for _ in range(world)]
        dev = [torch.from_numpy(p).cuda() for p in parts]
        dw = [torch.full((two_d,), float("nan"), device="cuda") for _ in range(world)]
        ds = [torch.full((C - two_d,), float("nan"), device="cuda") for _ in range(world)]
        ptrs = lambda ts: (ctypes.c_void_p * world)(*[t.data_ptr() for t in ts])  # noqa: E731
        st = lib.flash_prologue_peer_reduce_emulated(ptrs(dev), G, C, two_d, ptrs(dw), ptrs(ds),
                                                     ctypes.byref(desc), epoch, _lib.stream_of(torch.device("cuda")))
        assert st == 0
        torch.cuda.synchronize()
        local = [_finalize_order(p) for p in parts]
        total = local[0].copy()
        for v in local[1:]:
            total = (total + v).astype(np.float32)
        for r in range(world):
            got = np.concatenate((dw[r].cpu().numpy(), ds[r].cpu().numpy()))
            assert np.array_equal(got, total), (epoch, r)
    assert _lib.device_error(reset=True) == 0


def _c2_problem(seed=0, T=2048, H=16, D=64):
    g = torch.Generator(device="cuda").manual_seed(seed)
    buf = torch.randn(T, 3, H, D, generator=g, device="cuda").to(torch.bfloat16)
    q4, k4 = (buf[:, i].permute(1, 0, 2)[None] for i in (0, 1))
    gq, gk = (torch.randn(T, H, D, generator=g, device="cuda").to(torch.bfloat16).permute(1, 0, 2)[None]
              for _ in range(2))
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    ang = torch.rand(T, D // 2, generator=g, device="cuda") * 6
    return q4, k4, w, s, ang.sin(), ang.cos(), gq, gk


@pytest.mark.gpu
def test_bwd_dp_with_one_rank_equals_bwd():
    from flash_attn_prologue_b200.fused_epilogue import bwd_workspace_bytes, _get_compact_strides
    lib = _lib.load()
    q4, k4, w, s, sin, cos, gq, gk = _c2_problem()
    B, H, N, D = q4.shape
    datas, flags = _buffers(1, 160, "cuda")
    desc = _desc(1, 0, 160, datas, flags)
    ws = torch.empty(bwd_workspace_bytes(B, H, N, D, q4.dtype), dtype=torch.uint8, device="cuda")
    tab = _lib.strides3((0, D // 2, 1))
    outs = []
    for dp in (False, True, True):
        dq = torch.empty_strided(q4.shape, _get_compact_strides(q4.shape, q4.stride()), dtype=q4.dtype, device="cuda")
        dk = torch.empty_like(dq)
        dw, ds = torch.empty(2, 1, D, device="cuda"), torch.empty(H, 1, 1, device="cuda")
        args = (_lib.ptr(q4), _lib.strides4(q4), _lib.ptr(k4), _lib.strides4(k4), _lib.ptr(w), _lib.ptr(s),
                _lib.ptr(sin), tab, _lib.ptr(cos), tab, _lib.ptr(gq), _lib.strides4(gq), _lib.ptr(gk),
                _lib.strides4(gk), _lib.ptr(dq), _lib.strides4(dq), _lib.ptr(dk), _lib.strides4(dk),
                _lib.ptr(dw), _lib.ptr(ds), _lib.ptr(ws), ws.numel(), B, H, N, D, 1e-5, 0)
        stream = _lib.stream_of(q4.device)
        if dp:
            st = lib.flash_prologue_bwd_dp(*args, ctypes.byref(desc), len(outs), stream)
        else:
            st = lib.flash_prologue_bwd(*args, stream)
        assert st == 0
        outs.append((dq, dk, dw, ds))
    torch.cuda.synchronize()
    for dp_out in outs[1:]:
        for a, b in zip(outs[0], dp_out):
            assert torch.equal(_bits(a), _bits(b))
    assert _lib.device_error(reset=True) == 0


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _backward_paths(q4, k4, w, s, sin, cos, gq, gk):
    """Each prologue backward reachable from the public API: name -> f(use_group) -> grads."""
    from flash_attn_prologue_b200 import qknorm_rope_scale, qknorm_rope_scale_qkv
    q, k = q4[0].permute(1, 0, 2), k4[0].permute(1, 0, 2)
    g_q, g_k = gq[0].permute(1, 0, 2), gk[0].permute(1, 0, 2)

    def regular(ctx):
        args = [t.detach().clone().requires_grad_(i < 4) for i, t in enumerate((q, k, w, s, sin, cos))]
        out = qknorm_rope_scale(*args, backend="cute")
        with ctx():
            return torch.autograd.grad(out, args[:4], (g_q, g_k))

    def inverse(ctx):
        qq, kk = q4.detach().clone().requires_grad_(), k4.detach().clone().requires_grad_()
        ww, ss = w.detach().clone().requires_grad_(), s.detach().clone().requires_grad_()
        s4, c4 = (t[:, None].permute(1, 0, 2)[None] for t in (sin, cos))
        qo, ko, _, _ = torch.ops.flash_prologue.qknorm_rope_scale_cute_inverse(qq, kk, ww, ss, s4, c4, 1e-5)
        with ctx():
            return torch.autograd.grad((qo, ko), (qq, kk, ww, ss), (gq, gk))

    def packed(ctx):
        qkv = torch.stack((q, k, q), dim=1).detach().requires_grad_()
        ww, ss = w.detach().clone().requires_grad_(), s.detach().clone().requires_grad_()
        qo, ko, _ = qknorm_rope_scale_qkv(qkv, ww, ss, sin, cos)
        with ctx():
            return torch.autograd.grad((qo, ko), (qkv, ww, ss), (g_q, g_k))

    return {"regular": regular, "inverse": inverse, "packed": packed}


@pytest.mark.gpu
def test_every_backward_path_dispatches_to_the_group_in_a_one_rank_process_group():
    """Inside reducing(), every backward path calls its _dp entry (the group's epoch
    advances once per call) and a one-rank group returns the plain call's bits."""
    import contextlib
    import torch.distributed as dist
    from flash_attn_prologue_b200 import prepare_backend
    from flash_attn_prologue_b200.distributed import PeerGroup
    prepare_backend("cute")
    started = False
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ["MASTER_PORT"] = str(_free_port())
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", 0))
        started = True
    try:
        pg = PeerGroup(device=torch.device("cuda", 0), max_cols=2 * 64 + 16)
        paths = _backward_paths(*_c2_problem(seed=3))
        for n, (name, fn) in enumerate(paths.items(), start=1):
            plain = fn(contextlib.nullcontext)
            reduced = fn(pg.reducing)
            torch.cuda.synchronize()
            assert pg.epoch == n, name
            for a, b in zip(plain, reduced):
                assert torch.equal(_bits(a), _bits(b)), name
        assert _lib.device_error(reset=True) == 0
        pg.close()
    finally:
        if started:
            dist.destroy_process_group()


@pytest.mark.gpu
def test_rank_that_never_arrives_times_out_with_nan_and_error_word():
    """A two-rank group whose second rank never runs: the wait gives up after wait_ms.

    Both ranks' buffers are local and nothing plays rank 1, so its flag is
    never set: the kernel must stop waiting after 100 ms, write NaN, set the
    device error word, and leave the context usable for the next call.
    """
    import time
    lib = _lib.load()
    q4, k4, w, s, sin, cos, gq, gk = _c2_problem(seed=5, T=512)
    B, H, N, D = q4.shape
    from flash_attn_prologue_b200.fused_epilogue import bwd_workspace_bytes, _get_compact_strides
    datas, flags = _buffers(2, 160, "cuda")
    desc = _desc(2, 0, 160, datas, flags)
    desc.wait_ms = 100
    ws = torch.empty(bwd_workspace_bytes(B, H, N, D, q4.dtype), dtype=torch.uint8, device="cuda")
    tab = _lib.strides3((0, D // 2, 1))
    dq = torch.empty_strided(q4.shape, _get_compact_strides(q4.shape, q4.stride()), dtype=q4.dtype, device="cuda")
    dk = torch.empty_like(dq)
    dw, ds = torch.zeros(2, 1, D, device="cuda"), torch.zeros(H, 1, 1, device="cuda")
    args = (_lib.ptr(q4), _lib.strides4(q4), _lib.ptr(k4), _lib.strides4(k4), _lib.ptr(w), _lib.ptr(s),
            _lib.ptr(sin), tab, _lib.ptr(cos), tab, _lib.ptr(gq), _lib.strides4(gq), _lib.ptr(gk),
            _lib.strides4(gk), _lib.ptr(dq), _lib.strides4(dq), _lib.ptr(dk), _lib.strides4(dk),
            _lib.ptr(dw), _lib.ptr(ds), _lib.ptr(ws), ws.numel(), B, H, N, D, 1e-5, 0)
    assert _lib.device_error(reset=True) == 0
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert lib.flash_prologue_bwd_dp(*args, ctypes.byref(desc), 1, _lib.stream_of(q4.device)) == 0
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert 0.09 < elapsed < 5.0, elapsed
    assert torch.isnan(dw).all() and torch.isnan(ds).all()
    assert _lib.device_error(reset=True) != 0
    # the context is still usable: the plain backward runs and its gradients are finite
    assert lib.flash_prologue_bwd(*args, _lib.stream_of(q4.device)) == 0
    torch.cuda.synchronize()
    assert torch.isfinite(dw).all() and torch.isfinite(ds).all()
    assert _lib.device_error(reset=True) == 0


def _two_rank_worker(rank, world, port, steps, errq):
    """One rank: local backward, then the same backward inside PeerGroup.reducing()."""
    try:
        import torch.distributed as dist
        from flash_attn_prologue_b200 import prepare_backend, qknorm_rope_scale
        from flash_attn_prologue_b200.distributed import PeerGroup
        torch.cuda.set_device(rank)
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        prepare_backend("cute")
        pg = PeerGroup(device=torch.device("cuda", rank), max_cols=2 * 64 + 16, wait_ms=2000)
        for step in range(steps):
            q4, k4, w, s, sin, cos, gq, gk = _c2_problem(seed=100 * step + rank, T=1024 + 512 * rank)
            q, k = q4[0].permute(1, 0, 2), k4[0].permute(1, 0, 2)
            g_q, g_k = gq[0].permute(1, 0, 2), gk[0].permute(1, 0, 2)
            w, s = w.requires_grad_(), s.requires_grad_()
            out = qknorm_rope_scale(q, k, w, s, sin, cos, backend="cute")
            local = torch.autograd.grad(out, (w, s), (g_q, g_k), retain_graph=True)
            with pg.reducing():
                summed = torch.autograd.grad(out, (w, s), (g_q, g_k))
            flat_local = torch.cat([t.reshape(-1) for t in local])
            flat_sum = torch.cat([t.reshape(-1) for t in summed])
            every_local = [torch.empty_like(flat_local) for _ in range(world)]
            every_sum = [torch.empty_like(flat_sum) for _ in range(world)]
            dist.all_gather(every_local, flat_local)
            dist.all_gather(every_sum, flat_sum)
            expect = every_local[0].clone()
            for r in range(1, world):
                expect = expect + every_local[r]
            for r in range(world):  # every rank holds the same bits: the rank-order sum
                assert torch.equal(_bits(every_sum[r]), _bits(expect)), (step, r)
        assert pg.epoch == steps
        assert _lib.device_error(reset=True) == 0
        dist.barrier()
        pg.close()
        dist.destroy_process_group()
    except BaseException as e:  # noqa: BLE001 - reported to the parent
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.gpu
def test_peer_group_processes_on_every_visible_gpu():
    """One rank per visible GPU (2 to 8): the reduced gradients are the rank-order sum, bit for
    bit, on every rank, four steps in a row (both buffer halves, each reused)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import time
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    world, port = min(torch.cuda.device_count(), _lib.MAX_PEERS), _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, world, port, 4, errq)) for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.monotonic() + 240
    for p in procs:
        p.join(max(1.0, deadline - time.monotonic()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not alive, "ranks did not finish in time"
    assert not errors and all(p.exitcode == 0 for p in procs), (errors, [p.exitcode for p in procs])
