"""Data-parallel host logic on CPU ranks (gloo, world size 2).

Covers the only collective of the path: the sum over ranks of d rmsnorm_weight
and d scales (flash_attn_prologue_b200/distributed.py), in its deterministic
(all_gather + one column sum, identical bits on every rank) and all_reduce forms, the token sharding helper,
the sharded-equals-unsharded property of the whole forward/backward, and a
failure made on the host: a rank that leaves before the collective must make
its peer fail with an error instead of hanging.
"""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_attn_prologue_b200.distributed import reduce_param_grads, shard_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _worker_reduce(rank, world, port, out):
    try:
        _init(rank, world, port)
        g = torch.Generator().manual_seed(100 + rank)
        dw = torch.randn(2, 1, 64, generator=g)
        ds = torch.randn(16, 1, 1, generator=g)
        a = reduce_param_grads(dw, ds, deterministic=True)
        b = reduce_param_grads(dw, ds, deterministic=False)
        out.put((rank, a[0], a[1], b[0], b[1], None))
        dist.destroy_process_group()
    except Exception:
        out.put((rank, None, None, None, None, traceback.format_exc()))


def _run(target, world, *extra):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, out, *extra)) for r in range(world)]
    for p in procs:
        p.start()
    results = [out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(results, key=lambda r: r[0])


def test_param_grad_reduction_two_ranks():
    results = _run(_worker_reduce, 2)
    for r in results:
        assert r[-1] is None, r[-1]
    exp_dw = sum(torch.randn(2, 1, 64, generator=torch.Generator().manual_seed(100 + r))
                 for r in range(2))
    gens = [torch.Generator().manual_seed(100 + r) for r in range(2)]
    exp_ds = 0
    for g in gens:
        torch.randn(2, 1, 64, generator=g)
        exp_ds = exp_ds + torch.randn(16, 1, 1, generator=g)
    for rank, dw_det, ds_det, dw_ar, ds_ar, _ in results:
        # rank-order sum: bit-identical on every rank and equal to r0 + r1
        torch.testing.assert_close(dw_det, exp_dw, rtol=0, atol=0)
        torch.testing.assert_close(ds_det, exp_ds, rtol=0, atol=0)
        torch.testing.assert_close(dw_ar, exp_dw, rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(ds_ar, exp_ds, rtol=1e-6, atol=1e-6)
    assert torch.equal(results[0][1], results[1][1]) and torch.equal(results[0][2], results[1][2])


def _worker_three(rank, world, port, out):
    """Three ranks: the deterministic reduction gives the same bits on every rank, and
    ParamGradReducer (synchronous on CPU tensors) returns what reduce_param_grads does."""
    try:
        _init(rank, world, port)
        from flash_attn_prologue_b200.distributed import ParamGradReducer
        g = torch.Generator().manual_seed(200 + rank)
        dw = torch.randn(2, 1, 32, generator=g)
        ds = torch.randn(8, 1, 1, generator=g)
        a = reduce_param_grads(dw, ds)
        reducer = ParamGradReducer()
        b = reducer.reduce(dw, ds)
        reducer.wait()
        out.put((rank, a[0], a[1], b[0], b[1], None))
        dist.destroy_process_group()
    except Exception:
        out.put((rank, None, None, None, None, traceback.format_exc()))


def test_three_ranks_identical_bits_and_side_stream_reducer():
    results = _run(_worker_three, 3)
    for r in results:
        assert r[-1] is None, r[-1]
    exp_dw, exp_ds = 0, 0
    for r in range(3):
        g = torch.Generator().manual_seed(200 + r)
        exp_dw = exp_dw + torch.randn(2, 1, 32, generator=g)
        exp_ds = exp_ds + torch.randn(8, 1, 1, generator=g)
    for rank, dw, ds, rdw, rds, _ in results:
        assert torch.equal(dw, results[0][1]) and torch.equal(ds, results[0][2])
        assert torch.equal(rdw, dw) and torch.equal(rds, ds)
        torch.testing.assert_close(dw, exp_dw, rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(ds, exp_ds, rtol=1e-6, atol=1e-6)


def _worker_sharded(rank, world, port, out):
    """Each rank runs the native formulation on its token shard; reduced grads
    must equal the single-process result (the per-row op shards exactly)."""
    try:
        _init(rank, world, port)
        from oracle import native_forward
        T, H, D = 96, 4, 32
        g = torch.Generator().manual_seed(7)
        q = torch.randn(T, H, D, generator=g)
        k = torch.randn(T, H, D, generator=g)
        w = 1 + 0.1 * torch.randn(2, 1, D, generator=g)
        s = 0.1 * torch.randn(H, 1, 1, generator=g)
        ang = torch.randn(T, D // 2, generator=g)
        gq = torch.randn(T, H, D, generator=g)
        gk = torch.randn(T, H, D, generator=g)
        lo, hi = shard_range(T, rank, world, align=16)
        args = [x.clone().requires_grad_(i < 4) for i, x in
                enumerate((q[lo:hi], k[lo:hi], w, s, ang[lo:hi].sin(), ang[lo:hi].cos()))]
        outs = native_forward(*args)
        grads = torch.autograd.grad(outs, args[2:4], (gq[lo:hi], gk[lo:hi]))
        dw, ds = reduce_param_grads(grads[0], grads[1])
        full = [x.clone().requires_grad_(i < 4) for i, x in
                enumerate((q, k, w, s, ang.sin(), ang.cos()))]
        fouts = native_forward(*full)
        fgrads = torch.autograd.grad(fouts, full[2:4], (gq, gk))
        out.put((rank, float((dw - fgrads[0]).abs().max()), float((ds - fgrads[1]).abs().max()), None))
        dist.destroy_process_group()
    except Exception:
        out.put((rank, None, None, traceback.format_exc()))


def test_sharded_gradients_match_unsharded():
    for rank, edw, eds, err in _run(_worker_sharded, 2):
        assert err is None, err
        assert edw < 1e-4 and eds < 1e-4


def _worker_leaver(rank, world, port, out):
    """Rank 1 leaves between steps (before the collective); rank 0 must fail fast."""
    try:
        _init(rank, world, port, timeout_s=10)
        dist.barrier()
        if rank == 1:
            out.put((rank, "left", None))
            out.close()
            out.join_thread()  # flush the message before the abrupt exit
            os._exit(0)  # leaves without destroying the group: a lost peer
        try:
            reduce_param_grads(torch.zeros(2, 1, 8), torch.zeros(4, 1, 1))
            out.put((rank, "no error", None))
        except Exception as exc:  # gloo reports the lost peer or the timeout
            out.put((rank, "raised", type(exc).__name__))
    except Exception:
        out.put((rank, "setup failed", traceback.format_exc()))


def test_lost_rank_fails_the_collective_instead_of_hanging():
    results = _run(_worker_leaver, 2)
    assert results[1][1] == "left"
    assert results[0][1] == "raised", results[0]


@pytest.mark.parametrize("total,world,align", [(1 << 20, 8, 4096), (100, 3, 1), (7, 4, 4), (0, 2, 1)])
def test_shard_range_covers_exactly_once(total, world, align):
    covered = []
    for r in range(world):
        lo, hi = shard_range(total, r, world, align)
        assert lo <= hi
        if hi > lo:
            assert lo % align == 0
        covered.extend(range(lo, hi))
    assert covered == list(range(total))
