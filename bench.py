"""Benchmark of the attention prologue (forward + backward) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (benchmark configuration C2): packed forward + backward of
qknorm_rope_scale on q/k that are strided views of one BF16 QKV buffer
[T=1,048,576, 3, H=16, D=64], sin/cos FP32 [T, 32] (theta 10000, positions
restart every 4096 tokens), scales ~N(0, 0.1), upstream gradients ~N(0, 1).
One step = forward + backward over the T tokens of a rank (weak scaling: every
rank owns its own T-token shard) followed, at N > 1, by the data-parallel
reduction of d rmsnorm_weight / d scales over NCCL.

Metric: algorithmic HBM bytes per second of forward + backward (GB/s), plus
Mtokens/s and the fraction of 8 TB/s. Algorithmic bytes per token:
forward  H*D*2*4 + D*4 = 8,448 B (read q, k; write q_out, k_out; sin+cos row)
backward H*D*2*6 + D*4 = 12,544 B (read q, k, dq_out, dk_out; write dq, dk; sin+cos).
Inputs (6.4 GB buffer) exceed the 126 MB L2, so no flush is needed between steps.

``value`` is timed with CUDA events on the launching stream with inputs resident
in HBM; ``e2e`` adds, every step, the pinned host->device copy of the step's
inputs and the device->host copy of its outputs, through the same public API.
``--impl reference`` times the reference formulation (the CPU oracle port of
the reference ``native`` backend) on the host cores on a bounded token sample.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "prologue fwd+bwd HBM GB/s (% of 8 TB/s) and Mtokens/s at 1/2/4/8 B200"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
T_TOKENS, HEADS, HEAD_DIM = 1 << 20, 16, 64
THETA, RESET = 10000.0, 4096
FWD_BYTES_PER_TOKEN = HEADS * HEAD_DIM * 2 * 4 + HEAD_DIM * 4
BWD_BYTES_PER_TOKEN = HEADS * HEAD_DIM * 2 * 6 + HEAD_DIM * 4
# DRAM traffic per token, dram__bytes_read.sum + dram__bytes_write.sum of one
# ncu capture of each kernel at T = 131,072 (summary kept under profiles/),
# scaled to a launch by the tokens it processes. Writes still dirty in L2 when a
# kernel ends are not counted by the capture, so traffic reads slightly below
# the algorithmic bytes.
NCU_TRAFFIC_BYTES_PER_TOKEN = {"fwd": 8181, "bwd": 12370}
# sm__pipe_tensor_cycles_active (% of active cycles) of the fused QKV GEMM +
# prologue kernel in one ncu capture at C5's full size (summary kept under
# profiles/qkv_gemm_pair_c5_t65536.md).
NCU_C5_TENSOR_ACTIVE_PCT = 80.9


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples over a marked region (warm-up + timed steps).

    The sampler process starts (and has produced its first sample) before the
    region begins, a reader thread timestamps every line, and the summary keeps
    the samples that arrived between ``begin()`` and ``end()``.
    """
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index, period_ms=20):
        self.index = index
        self.period_ms = period_ms
        self.proc = None
        self.samples = []
        self.t0 = self.t1 = None

    def __enter__(self):
        import threading
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", str(self.period_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return self
        first = threading.Event()

        def reader():
            for ln in self.proc.stdout:
                if ln.strip():
                    self.samples.append((time.perf_counter(), ln))
                    first.set()

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        first.wait(timeout=5.0)
        return self

    def begin(self):
        self.t0 = time.perf_counter()

    def end(self):
        self.t1 = time.perf_counter()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(2 * self.period_ms / 1000.0)  # the sample covering the region's end
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.thread.join(timeout=5)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        t0 = self.t0 if self.t0 is not None else -1e30
        t1 = (self.t1 if self.t1 is not None else 1e30) + self.period_ms / 1000.0
        for ts, ln in self.samples:
            if not (t0 <= ts <= t1):
                continue
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        window = round((self.t1 - self.t0) * 1e3, 1) if self.t0 is not None and self.t1 is not None else None
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "window_ms": window}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "window_ms": window}


def rope_tables(positions, d, theta):
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64, device=positions.device) / d))
    ang = (positions.double()[:, None] * inv[None]).float()
    return ang.sin(), ang.cos()


def make_inputs(T, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    buf = torch.randn(T, 3, HEADS, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
    pos = torch.arange(T, device=device) % RESET
    sin, cos = rope_tables(pos, HEAD_DIM, THETA)
    w = 1 + 0.02 * torch.randn(2, 1, HEAD_DIM, generator=g, device=device)
    s = 0.1 * torch.randn(HEADS, 1, 1, generator=g, device=device)
    gq = torch.randn(T, HEADS, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
    gk = torch.randn(T, HEADS, HEAD_DIM, generator=g, device=device).to(torch.bfloat16)
    return buf, w, s, sin, cos, gq, gk


def dist_setup(args):
    """One process per GPU (torchrun env); NCCL process group for our arm at N > 1."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local if world > 1 else 0)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(value, world):
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_sample_run(tokens, reps, threads):
    """Times the reference formulation (oracle port of ``native``) on host cores."""
    from oracle import native_forward
    torch.set_num_threads(threads)
    buf, w, s, sin, cos, gq, gk = make_inputs(tokens, "cpu", 7)
    q, k = buf[:, 0], buf[:, 1]
    times = []
    for i in range(reps + 1):
        args = [t.detach().requires_grad_(j < 4) for j, t in enumerate((q, k, w, s, sin, cos))]
        t0 = time.perf_counter()
        out = native_forward(*args)
        torch.autograd.grad(out, args[:4], (gq, gk))
        dt = time.perf_counter() - t0
        if i > 0:  # first call warms up
            times.append(dt)
    per_call = statistics.median(times)
    gbs = tokens * (FWD_BYTES_PER_TOKEN + BWD_BYTES_PER_TOKEN) / per_call / 1e9
    return gbs, per_call


def run_reference(args, world, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    tokens = args.cpu_tokens
    times = []
    for _ in range(args.warmup):
        cpu_sample_run(tokens, 1, threads)
    for _ in range(args.steps):
        _, per = cpu_sample_run(tokens, 1, threads)
        times.append(per)
    per = statistics.median(times)
    gbs = tokens * (FWD_BYTES_PER_TOKEN + BWD_BYTES_PER_TOKEN) / per / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "mtokens_per_s": round(tokens / per / 1e6, 4),
        "config": {"workload": f"C2 packed fwd+bwd, {tokens}-token sample of T=1,048,576, "
                               f"H={HEADS}, D={HEAD_DIM}, strided views of a [T,3,H,D] BF16 buffer",
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{tokens} tokens of C2 per step (fwd+bwd), torch eager CPU"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def min_over_ranks(value, world):
    return -max_over_ranks(-value, world)


def _timed_loop(fn, steps, warmup, world, finish=None):
    """Barrier + synchronize on both sides of `steps` calls of fn(); device time (ms) per
    call, max over ranks. fn runs on the current stream (and may fork work off it);
    finish() joins forked work into the current stream before the end event."""
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        fn()
    if finish is not None:
        finish()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    if finish is not None:
        finish()
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(start.elapsed_time(end), world) / steps


def run_ours(args, world, rank, local):
    from flash_attn_prologue_b200 import prepare_backend, qknorm_rope_scale
    from flash_attn_prologue_b200.distributed import ParamGradReducer, PeerGroup
    prepare_backend("cute")
    device = torch.device("cuda", torch.cuda.current_device())
    T = args.tokens
    buf, w, s, sin, cos, gq, gk = make_inputs(T, device, 1234 + rank)
    q, k = buf[:, 0], buf[:, 1]
    w.requires_grad_()
    s.requires_grad_()

    stream = torch.cuda.current_stream()
    peer = args.dp_reduce == "peer" and world > 1
    reducer = ParamGradReducer(device=device) if world > 1 and not peer else None
    peers = PeerGroup(device=device, max_cols=2 * HEAD_DIM + HEADS) if peer else None
    fwd_ev, bwd_ev, coll_ev = [], [], []

    def step(record=False):
        qq = q.detach().requires_grad_()
        kk = k.detach().requires_grad_()
        if record:
            e0 = torch.cuda.Event(enable_timing=True); e0.record(stream)
        out = qknorm_rope_scale(qq, kk, w, s, sin, cos, backend="cute")
        if record:
            e1 = torch.cuda.Event(enable_timing=True); e1.record(stream)
        if peers is not None:
            # d w / d s come out of the backward already summed over the ranks
            with peers.reducing():
                dq, dk, dw, ds = torch.autograd.grad(out, (qq, kk, w, s), (gq, gk))
        else:
            dq, dk, dw, ds = torch.autograd.grad(out, (qq, kk, w, s), (gq, gk))
        if record:
            e2 = torch.cuda.Event(enable_timing=True); e2.record(stream)
            fwd_ev.append((e0, e1))
            bwd_ev.append((e1, e2))
        if reducer is not None:
            # The parameter-gradient reduction on a side stream, overlapping the
            # next step's forward; its events time it on that stream.
            if record:
                c0 = torch.cuda.Event(enable_timing=True)
                c1 = torch.cuda.Event(enable_timing=True)
                reducer.stream.wait_stream(stream)
                c0.record(reducer.stream)
            dw, ds = reducer.reduce(dw, ds)
            if record:
                c1.record(reducer.stream)
                coll_ev.append((c0, c1))
        return out, dq, dk, dw, ds

    with ClockSampler(local) as clocks:
        clocks.begin()
        for _ in range(args.warmup):
            step()
        if reducer is not None:
            reducer.wait()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            step(record=True)
        if reducer is not None:
            reducer.wait()  # the last reduction is part of the timed work
        end.record(stream)
        torch.cuda.synchronize()
        clocks.end()
    barrier(world)
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world)
    fwd_ms = statistics.mean(a.elapsed_time(b) for a, b in fwd_ev)
    bwd_ms = statistics.mean(a.elapsed_time(b) for a, b in bwd_ev)
    fwd_ms, bwd_ms = max_over_ranks(fwd_ms, world), max_over_ranks(bwd_ms, world)

    ms_per_step = elapsed_ms / args.steps
    step_bytes = T * (FWD_BYTES_PER_TOKEN + BWD_BYTES_PER_TOKEN)
    value = world * step_bytes / (ms_per_step * 1e-3) / 1e9
    mtok = world * T / (ms_per_step * 1e-3) / 1e6
    peak, peak_kind = measured_peak()

    coll = None
    if peers is not None:
        from flash_attn_prologue_b200 import _lib
        peer_error = int(max_over_ranks(float(_lib.device_error(reset=True)), world))
        coll = {"how": "in the backward's finalize kernel: each rank's [2*D+H] sums written to every "
                       "rank's exchange buffer over NVLink, flags, rank-order sum (bwd.ms includes it)",
                "isolated_ms": round(isolated_peer_reduction_ms(device, world, peers), 4),
                "floats": 2 * HEAD_DIM + HEADS, "device_error": peer_error}
    elif world > 1:
        # The reduction alone: on its side stream inside the step (from the end of
        # the backward to the sum's completion, so it includes waiting for the
        # slowest rank), and isolated (back-to-back on the main stream).
        side = [a.elapsed_time(b) for a, b in coll_ev]
        coll = {"in_step_ms": round(max_over_ranks(statistics.mean(side), world), 4),
                "in_step_max_ms": round(max_over_ranks(max(side), world), 4),
                "isolated_ms": round(isolated_reduction_ms(device, world), 4),
                "floats": 2 * HEAD_DIM + HEADS,
                "how": "pack + NCCL all_gather + column sum on a side stream; in_step spans the "
                       "end of the backward to the sum (it waits while the next forward holds the SMs)"}
    del buf, gq, gk
    if peers is not None:
        barrier(world)
        peers.close()

    c4 = run_c4(args, device, world, rank, peak)
    c3 = run_c3(args, device, world, rank, peak)

    # ---- end to end: host buffers through the public API, copies timed ----
    e2e = run_e2e(args, T, device, w, s, world, local)

    bwd_gbs = T * BWD_BYTES_PER_TOKEN / (bwd_ms * 1e-3) / 1e9
    fwd_gbs = T * FWD_BYTES_PER_TOKEN / (fwd_ms * 1e-3) / 1e9
    traffic = NCU_TRAFFIC_BYTES_PER_TOKEN["bwd"]
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"C2 packed fwd+bwd, T={T} tokens per GPU, H={HEADS}, D={HEAD_DIM}, "
                               "q/k strided views of a [T,3,H,D] BF16 buffer",
                   "l2": "inputs > L2 (6.4 GB per GPU), no flush", "parallelism": f"dp{world}"},
        "mtokens_per_s": round(mtok, 3),
        "pct_of_8tbs": round(100 * value / world / NOMINAL_HBM_GBS, 2),
        "fwd": {"ms": round(fwd_ms, 4), "gbs": round(fwd_gbs, 1), "frac": round(fwd_gbs / peak, 4)},
        "bwd": {"ms": round(bwd_ms, 4), "gbs": round(bwd_gbs, 1), "frac": round(bwd_gbs / peak, 4)},
        "roofline": {"kernel": "prologue_bwd_tma_kernel+finalize", "bound": "hbm",
                     "achieved": round(bwd_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(bwd_gbs / peak, 4), "peak_source": peak_kind,
                     "traffic": (round(traffic * T) if traffic else None),
                     "traffic_src": "ncu at T=131072, x8 to T"},
        "collective": coll, "c3": c3, "c4": c4,
        "e2e": e2e,
        "gpu_launches": 3 * args.steps,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        gbs, per = cpu_sample_run(args.cpu_tokens, args.cpu_reps, threads)
        line["cpu_baseline"] = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                                "kind": "port",
                                "sample": f"{args.cpu_tokens} tokens of C2 fwd+bwd, median of "
                                          f"{args.cpu_reps}, torch eager CPU port of native"}
    if rank == 0 and world == 1 and not args.no_extras:
        line["x"] = run_extras(device, peak)
    if rank == 0:
        print(json.dumps(line, separators=(",", ":")), flush=True)
    if args.detail and rank == 0:
        Path(args.detail).write_text(json.dumps(line, indent=1))


def isolated_peer_reduction_ms(device, world, peers, reps=20):
    """Device time of a 16-token backward inside peers.reducing() (its backward kernel
    takes a few microseconds; the rest is the peer finalize), ranks aligned by a barrier
    before each call."""
    from flash_attn_prologue_b200 import qknorm_rope_scale
    T = 16
    buf, w, s, sin, cos, gq, gk = make_inputs(T, device, 7)
    w.requires_grad_()
    s.requires_grad_()
    times = []
    for i in range(reps + 3):
        out = qknorm_rope_scale(buf[:, 0], buf[:, 1], w, s, sin, cos, backend="cute")
        torch.cuda.synchronize()
        barrier(world)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        with peers.reducing():
            torch.autograd.grad(out, (w, s), (gq, gk))
        b.record()
        torch.cuda.synchronize()
        if i >= 3:
            times.append(a.elapsed_time(b))
    return max_over_ranks(statistics.median(times), world)


def isolated_reduction_ms(device, world, reps=20):
    """Device time of one reduce_param_grads call (pack, all_gather, sum) on an idle GPU:
    the stream is held by a spin kernel while the host enqueues the call, so the
    three kernels run back to back and the host's enqueue time is not measured;
    median over reps, max over ranks."""
    from flash_attn_prologue_b200.distributed import reduce_param_grads
    dw0 = torch.randn(2, 1, HEAD_DIM, device=device)
    ds0 = torch.randn(HEADS, 1, 1, device=device)
    for _ in range(3):
        reduce_param_grads(dw0, ds0)
    times = []
    for _ in range(reps):
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda._sleep(2_000_000)  # ~1 ms: covers the host's enqueue of the call
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        reduce_param_grads(dw0, ds0)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return max_over_ranks(statistics.median(times), world)


def run_c4(args, device, world, rank, peak):
    """C4: packed backward of T=262,144 tokens (H=8, D=64) per rank, then the
    reduction of d rmsnorm_weight / d scales over the ranks (weak scaling)."""
    from flash_attn_prologue_b200.distributed import ParamGradReducer
    T, H, D = 262144, 8, 64
    g = torch.Generator(device=device).manual_seed(40 + rank)
    q, k, gq, gk = (torch.randn(T, H, D, generator=g, device=device).to(torch.bfloat16)
                    for _ in range(4))
    sin, cos = rope_tables(torch.arange(T, device=device), D, 10000.0)
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device=device)
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device=device)
    bwd = torch.ops.flash_prologue.qknorm_rope_scale_cute_backward
    q4, k4 = q.permute(1, 0, 2)[None], k.permute(1, 0, 2)[None]
    g4q, g4k = gq.permute(1, 0, 2)[None], gk.permute(1, 0, 2)[None]
    s4 = sin[None, None].expand(1, 1, T, D // 2)
    c4 = cos[None, None].expand(1, 1, T, D // 2)
    reducer = ParamGradReducer(device=device) if world > 1 else None

    def step():
        dq, dk, dw, ds = bwd(q4, k4, w, s, s4, c4, g4q, g4k, 1e-5)
        if reducer is not None:
            reducer.reduce(dw, ds)

    def join():
        if reducer is not None:
            reducer.wait()

    def step_serial():
        step()
        join()

    # Each step's reduction overlaps the next step's backward (the last one is
    # joined inside the timing); "ms_serial" waits for every reduction in turn.
    ms = _timed_loop(step, args.steps, args.warmup, world, finish=join)
    ms_serial = _timed_loop(step_serial, args.steps, args.warmup, world)
    nbytes = T * (H * D * 2 * 6 + D * 4)
    gbs = world * nbytes / (ms * 1e-3) / 1e9
    return {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac": round(gbs / world / peak, 4),
            "ms_serial": round(ms_serial, 4), "tokens_per_gpu": T, "scaling": "weak"}


def run_c3(args, device, world, rank, peak):
    """C3: dense forward [B=8, H=32, S=8192, D=128], the batch sharded over the
    ranks (strong scaling: the whole problem's bytes over the slowest rank's time)."""
    from flash_attn_prologue_b200 import qknorm_rope_scale
    from flash_attn_prologue_b200.distributed import shard_range
    B, H, S, D = 8, 32, 8192, 128
    b0, b1 = shard_range(B, rank, world)
    g = torch.Generator(device=device).manual_seed(30 + rank)
    q, k = (torch.randn(b1 - b0, H, S, D, generator=g, device=device).to(torch.bfloat16) for _ in range(2))
    sin, cos = rope_tables(torch.arange(S, device=device), D, 500000.0)
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device=device)
    s = torch.full((H, 1, 1), math.log(1 / math.sqrt(D)), device=device)
    ms = _timed_loop(lambda: qknorm_rope_scale(q, k, w, s, sin, cos, backend="cute"),
                     args.steps, args.warmup, world)
    nbytes = B * H * S * D * 2 * 4 + S * D * 4
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac": round(gbs / world / peak, 4),
            "batches_per_gpu": b1 - b0, "scaling": "strong"}


def _event_ms(fn, steps, warmup=3):
    """Mean CUDA-event time of fn() on the current stream (inputs resident in HBM)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def run_extras(device, peak, steps=20):
    """The other single-GPU measurements, compact (reported beside the headline at N = 1).

    c1: C1 packed fwd [4096, 4, 32] eager and as one CUDA-graph replay.
    inv: C2 through the inverse formulation (fwd also stores r; bwd rebuilds rows).
    qkv_step: C2 training step to the [T, 3, H, D] gradient, through slice views
      + autograd gather, and through qknorm_rope_scale_qkv.
    c5: fused QKV GEMM + prologue, X [65536, 2048] x W [6144, 2048] (H=16, D=128):
      burst (`steps` launches) and sustained (450 launches, power-capped clocks)
      times of the fused kernel, the same kernel without the prologue, cuBLAS
      F.linear alone and F.linear + this prologue kernel; fractions against the
      measured bf16_tflops (burst) and bf16_tflops_sustained.
    c5_bwd: projection backward dX / dW kernels (gradients read in place), cuBLAS on
      an already gathered [T, 3HD] dP, and that gather.
    c5_step: forward + backward to x, W, rmsnorm_weight, scales: fused op vs
      F.linear + qknorm_rope_scale + autograd (cuBLAS).
    """
    import flash_attn_prologue_b200 as fap
    from flash_attn_prologue_b200 import qknorm_rope_scale
    out = {}
    g = torch.Generator(device=device).manual_seed(5)
    bf16_peak = _measured("bf16_tflops", 1590.0)
    r4 = lambda v: round(v, 4)  # noqa: E731

    def frac(nbytes, ms):
        return r4(nbytes / (ms * 1e-3) / 1e9 / peak)

    # C1
    T, H, D = 4096, 4, 32
    q, k = (torch.randn(T, H, D, generator=g, device=device).to(torch.bfloat16) for _ in range(2))
    sin, cos = rope_tables(torch.arange(T, device=device), D, 10000.0)
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device=device)
    s = torch.zeros(H, 1, 1, device=device)
    eager = _event_ms(lambda: qknorm_rope_scale(q, k, w, s, sin, cos, backend="cute"), steps)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        qknorm_rope_scale(q, k, w, s, sin, cos, backend="cute")
    out["c1"] = {"ms": r4(eager), "graph_ms": r4(_event_ms(graph.replay, max(steps, 200)))}
    del graph
    # C2 through the inverse formulation: strided views of the [T, 3, H, D]
    # buffer, algorithmic bytes + 4 B per row of r.
    T, H, D = T_TOKENS, HEADS, HEAD_DIM
    buf = torch.randn(T, 3, H, D, generator=g, device=device).to(torch.bfloat16)
    q4, k4 = (buf[:, i].permute(1, 0, 2)[None] for i in (0, 1))
    g4q, g4k = (torch.randn(T, H, D, generator=g, device=device).to(torch.bfloat16).permute(1, 0, 2)[None]
                for _ in range(2))  # packed [T, H, D] upstream gradients, like the outputs
    sin, cos = rope_tables(torch.arange(T, device=device) % 4096, D, 10000.0)
    s4, c4 = sin[None, None], cos[None, None]
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device=device)
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device=device)
    inv_fwd = torch.ops.flash_prologue.qknorm_rope_scale_cute_inverse
    inv_bwd = torch.ops.flash_prologue.qknorm_rope_scale_cute_inverse_backward
    qo, ko, rq, rk = inv_fwd(q4, k4, w, s, s4, c4, 1e-5)
    f_ms = _event_ms(lambda: inv_fwd(q4, k4, w, s, s4, c4, 1e-5), steps)
    b_ms = _event_ms(lambda: inv_bwd(qo, ko, w, s, s4, c4, g4q, g4k, rq, rk, 1e-5), steps)
    out["inv"] = {"fwd_ms": r4(f_ms), "fwd_frac": frac(T * (FWD_BYTES_PER_TOKEN + 2 * H * 4), f_ms),
                  "bwd_ms": r4(b_ms), "bwd_frac": frac(T * (BWD_BYTES_PER_TOKEN + 2 * H * 4), b_ms)}
    del q4, k4, qo, ko, rq, rk
    # C2 training step with the QKV gradient (V's gradient included).
    gq3, gk3 = (t[0].permute(1, 0, 2) for t in (g4q, g4k))
    gv3 = torch.randn(T, H, D, generator=g, device=device).to(torch.bfloat16)

    def step_slices():
        x = buf.detach().requires_grad_()
        q, k, v = x.unbind(1)
        qo_, ko_ = qknorm_rope_scale(q, k, w, s, sin, cos, backend="cute")
        return torch.autograd.grad((qo_, ko_, v), x, (gq3, gk3, gv3))

    def step_packed():
        x = buf.detach().requires_grad_()
        qo_, ko_, v = fap.qknorm_rope_scale_qkv(x, w, s, sin, cos)
        return torch.autograd.grad((qo_, ko_, v), x, (gq3, gk3, gv3))

    step_bytes = T * (FWD_BYTES_PER_TOKEN + BWD_BYTES_PER_TOKEN + H * D * 2 * 2)  # + dv read/write
    sl_ms, pk_ms = _event_ms(step_slices, steps), _event_ms(step_packed, steps)
    out["qkv_step"] = {"slices_ms": r4(sl_ms), "packed_ms": r4(pk_ms), "packed_frac": frac(step_bytes, pk_ms)}
    del buf, g4q, g4k, gq3, gk3, gv3
    # C5
    T, hidden, H, D = 65536, 2048, 16, 128
    x = torch.randn(1, T, hidden, generator=g, device=device).to(torch.bfloat16)
    wq = (0.02 * torch.randn(3 * H * D, hidden, generator=g, device=device)).to(torch.bfloat16)
    sin, cos = rope_tables(torch.arange(T, device=device), D, 10000.0)
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device=device)
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device=device)
    flop = 2 * T * 3 * H * D * hidden

    def unfused():
        p = torch.nn.functional.linear(x[0], wq).view(T, 3, H, D)
        return qknorm_rope_scale(p[:, 0], p[:, 1], w, s, sin, cos, backend="cute")

    fns = (("fused", lambda: fap.fused_qkv_epilogue(x, wq, w, s, sin, cos)),
           ("gemm_only", lambda: fap.fused_qkv(x, wq)),
           ("cublas", lambda: torch.nn.functional.linear(x[0], wq)),
           ("cublas_prologue", unfused))
    sustained_peak = _measured("bf16_tflops_sustained", 1410.0)
    c5 = {}
    # Burst: `steps` launches; sustained: ~0.6 s of back-to-back launches, where
    # the 1 kW power cap sets the clocks (the regime of a long training run).
    for regime, n, pk in (("", steps, bf16_peak), ("sus_", 450, sustained_peak)):
        ms = {name: _event_ms(fn, n) for name, fn in fns}
        tf = flop / (ms["fused"] * 1e-3) / 1e12
        if not regime:
            c5["tflops"] = round(tf, 1)
        c5[f"{regime}frac"] = r4(tf / pk)
        c5.update({f"{regime}{name}_ms": r4(v) for name, v in ms.items()})
    c5["ncu_tensor_active_pct"] = NCU_C5_TENSOR_ACTIVE_PCT
    out["c5"] = c5
    # C5 projection backward: dX = dP W and dW = dP^T X with dP the per-head
    # [1, H, T, D] gradients, by the hand-written kernels (read in place) and
    # by cuBLAS on an already gathered [T, 3HD] dP.
    gq5, gk5, gv5 = (torch.randn(1, H, T, D, generator=g, device=device).to(torch.bfloat16) for _ in range(3))

    def gather():
        return torch.stack((gq5, gk5, gv5), 0).permute(1, 3, 0, 2, 4).reshape(T, 3 * H * D).contiguous()

    dp = gather()
    x2 = x[0]
    ms = {name: _event_ms(fn, steps) for name, fn in (
        ("dx", lambda: fap.matmul_bwd_dx(gq5, gk5, gv5, wq)),
        ("dw", lambda: fap.matmul_bwd_dw(gq5, gk5, gv5, x)),
        ("cublas_dx", lambda: dp @ wq),
        ("cublas_dw", lambda: dp.t() @ x2),
        ("gather", gather))}
    c5b = {f"{k}_ms": r4(v) for k, v in ms.items()}
    for k in ("dx", "dw"):
        c5b[f"{k}_frac"] = r4(flop / (ms[k] * 1e-3) / 1e12 / bf16_peak)
    out["c5_bwd"] = c5b
    del dp
    # C5 training step: forward + backward to x, W, rmsnorm_weight and scales.
    xg = x.detach().requires_grad_()
    wg = wq.detach().requires_grad_()
    wr = w.detach().requires_grad_()
    sr = s.detach().requires_grad_()
    ups = (gq5, gk5, gv5)

    def step_fused():
        q_, k_, v_, _, _ = fap.fused_qkv_epilogue(xg, wg, wr, sr, sin, cos)
        return torch.autograd.grad((q_, k_, v_), (xg, wg, wr, sr), ups)

    def step_composed():
        p = torch.nn.functional.linear(xg, wg).view(1, T, 3, H, D)
        q_, k_ = qknorm_rope_scale(p[:, :, 0].transpose(1, 2), p[:, :, 1].transpose(1, 2), wr, sr, sin, cos,
                                   backend="cute")
        return torch.autograd.grad((q_, k_, p[:, :, 2].transpose(1, 2)), (xg, wg, wr, sr), ups)

    out["c5_step"] = {"fused_ms": r4(_event_ms(step_fused, steps)),
                      "composed_ms": r4(_event_ms(step_composed, steps))}
    del gq5, gk5, gv5, xg, wg
    return out


def _measured(key, fallback):
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())[key])
    except Exception:
        return fallback


def run_e2e(args, T, device, w, s, world, local):
    """Same metric with pinned host buffers: H2D inputs + D2H outputs inside the timing.

    Every step copies its inputs host->device, runs the public API forward +
    autograd backward, and copies all outputs and gradients device->host. Steps
    are pipelined over two device buffer sets and three streams, as a training
    loop with a prefetching loader would run them: step i+1's inputs upload while
    step i computes and its results download, so the two PCIe directions overlap.
    """
    from flash_attn_prologue_b200 import qknorm_rope_scale
    g = torch.Generator().manual_seed(99)
    tok = min(T, args.e2e_tokens)
    host_in = [torch.randn(tok, HEADS, HEAD_DIM, generator=g).to(torch.bfloat16).pin_memory()
               for _ in range(4)]  # q, k, grad q_out, grad k_out
    sin, cos = rope_tables(torch.arange(tok) % RESET, HEAD_DIM, THETA)
    host_in += [sin.pin_memory(), cos.pin_memory()]
    nbuf = 2
    dev_in = [[torch.empty(t.shape, dtype=t.dtype, device=device) for t in host_in] for _ in range(nbuf)]
    out_shapes = [((tok, HEADS, HEAD_DIM), torch.bfloat16)] * 4 + [((2, 1, HEAD_DIM), torch.float32),
                                                                   ((HEADS, 1, 1), torch.float32)]
    host_out = [[torch.empty(sh, dtype=dt).pin_memory() for sh, dt in out_shapes] for _ in range(nbuf)]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out[0])
    s_in, s_comp, s_out = (torch.cuda.Stream(device) for _ in range(3))
    comp_done = [torch.cuda.Event() for _ in range(nbuf)]
    in_done = [torch.cuda.Event() for _ in range(nbuf)]

    def step(i):
        b = i % nbuf
        with torch.cuda.stream(s_in):
            s_in.wait_event(comp_done[b])  # the compute that last read this buffer set is done
            for d, h in zip(dev_in[b], host_in):
                d.copy_(h, non_blocking=True)
            in_done[b].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(in_done[b])
            q, k = (t.detach().requires_grad_() for t in dev_in[b][:2])
            gq, gk, sn, cs = dev_in[b][2:]
            out = qknorm_rope_scale(q, k, w, s, sn, cs, backend="cute")
            dq, dk, dw, ds = torch.autograd.grad(out, (q, k, w, s), (gq, gk))
            results = (out[0], out[1], dq, dk, dw, ds)
            comp_done[b].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[b])
            for dst, src in zip(host_out[b], results):
                dst.copy_(src, non_blocking=True)
                src.record_stream(s_out)

    for i in range(2):
        step(i)
    torch.cuda.synchronize()
    barrier(world)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    steps = max(2, min(args.steps, 16))
    start.record(s_in)
    for i in range(steps):
        step(i)
    end.record(s_out)
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world) / steps
    gbs = world * tok * (FWD_BYTES_PER_TOKEN + BWD_BYTES_PER_TOKEN) / (ms * 1e-3) / 1e9
    # What bounds it: this rank's pinned-host copy bandwidth in each direction
    # alone (the step's own upload / download bytes, one direction at a time),
    # min over ranks, and where the GPU sits (its NUMA node).
    up = _copy_gbs(dev_in[0], host_in, steps=3)
    down = _copy_gbs(host_out[0], [t for t in dev_in[0][:4]] + [w.detach().reshape(-1), s.detach().reshape(-1)],
                     steps=3, to_host=True)
    return {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 3), "tokens_per_step": tok,
            "h2d_gbs_min": round(min_over_ranks(up, world), 1),
            "d2h_gbs_min": round(min_over_ranks(down, world), 1),
            "numa_node": _numa_node(local),
            "path": "public API, pinned host buffers, 2 buffer sets, H2D/compute/D2H on 3 streams"}


def _copy_gbs(dsts, srcs, steps=3, to_host=False):
    """GB/s of copying srcs into dsts (one direction), CUDA events on the current stream."""
    nbytes = sum(t.numel() * t.element_size() for t in (srcs if not to_host else dsts))
    pairs = list(zip(dsts, srcs))

    def run():
        for d, h in pairs:
            if d.numel() == h.numel():
                d.view(-1).copy_(h.reshape(-1), non_blocking=True)

    ms = _event_ms(run, steps, warmup=1)
    return nbytes / (ms * 1e-3) / 1e9


def _numa_node(local):
    """NUMA node of the GPU's PCI device (sysfs), or None."""
    try:
        out = subprocess.run(["nvidia-smi", f"--id={local}", "--query-gpu=pci.bus_id",
                              "--format=csv,noheader"], capture_output=True, text=True, timeout=10)
        bus = out.stdout.strip()
        bus = bus.lower()
        if bus.count(":") == 2 and len(bus.split(":")[0]) == 8:
            bus = bus[4:]  # 00000000:18:00.0 -> 0000:18:00.0
        return int(Path(f"/sys/bus/pci/devices/{bus}/numa_node").read_text().strip())
    except Exception:
        return None


def run_c5_profile_case(T):
    """Three launches of the fused QKV GEMM + prologue at C5's hidden size and heads."""
    import flash_attn_prologue_b200 as fap
    from flash_attn_prologue_b200 import _lib
    hidden, H, D = 2048, 16, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(1, T, hidden, generator=g, device="cuda").to(torch.bfloat16)
    wq = (0.02 * torch.randn(3 * H * D, hidden, generator=g, device="cuda")).to(torch.bfloat16)
    sin, cos = rope_tables(torch.arange(T, device="cuda"), D, 10000.0)
    w = 1 + 0.02 * torch.randn(2, 1, D, generator=g, device="cuda")
    s = 0.1 * torch.randn(H, 1, 1, generator=g, device="cuda")
    for _ in range(3):
        fap.fused_qkv_epilogue(x, wq, w, s, sin, cos)
    torch.cuda.synchronize()
    if _lib.device_error(reset=True) != 0:
        raise SystemExit("device error word set")


def run_c5_bwd_profile_case(T):
    """Three calls of the projection backward (dX and dW GEMM kernels) at C5's hidden size and heads."""
    import flash_attn_prologue_b200 as fap
    from flash_attn_prologue_b200 import _lib
    hidden, H, D = 2048, 16, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(1, T, hidden, generator=g, device="cuda").to(torch.bfloat16)
    wq = (0.02 * torch.randn(3 * H * D, hidden, generator=g, device="cuda")).to(torch.bfloat16)
    gq, gk, gv = (torch.randn(1, H, T, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    for _ in range(3):
        fap.fused_qkv_backward(gq, gk, gv, wq, x)
    torch.cuda.synchronize()
    if _lib.device_error(reset=True) != 0:
        raise SystemExit("device error word set")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=T_TOKENS, help="tokens per GPU (default: C2)")
    ap.add_argument("--e2e-tokens", type=int, default=T_TOKENS // 4)
    ap.add_argument("--cpu-tokens", type=int, default=32768)
    ap.add_argument("--cpu-reps", type=int, default=5)
    ap.add_argument("--dp-reduce", choices=["nccl", "peer"], default="nccl",
                    help="N > 1: sum d rmsnorm_weight / d scales with NCCL on a side stream, or "
                         "inside the backward's finalize kernel over NVLink peer memory")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the C1/inverse/QKV-step/C5 timings reported beside the headline")
    ap.add_argument("--store", choices=["auto", "tma", "lane"], default="auto",
                    help="how the pipelined prologue kernels store their outputs: the library's "
                         "measured choice (default), always TMA tensor stores, or the lanes' "
                         "16-byte stores (for profiling one form at a size where auto picks the other)")
    ap.add_argument("--detail", default="", help="also write the JSON line, indented, to this file")
    ap.add_argument("--c5-profile-tokens", type=int, default=0,
                    help="only run the fused QKV GEMM + prologue (C5 shapes, this many tokens) three "
                         "times and exit: the small case an ncu capture of that kernel uses")
    ap.add_argument("--c5-bwd-profile-tokens", type=int, default=0,
                    help="only run the projection backward GEMMs (C5 shapes, this many tokens) three "
                         "times: the case the backward GEMM ncu captures use")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.c5_profile_tokens:
        run_c5_profile_case(args.c5_profile_tokens)
        return
    if args.c5_bwd_profile_tokens:
        run_c5_bwd_profile_case(args.c5_bwd_profile_tokens)
        return
    if args.impl == "reference":
        # The reference path is CPU code: rank 0 runs it, other ranks exit at once.
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args)
    if args.store != "auto":
        from flash_attn_prologue_b200 import _lib
        _lib.set_path({"tma": 2, "lane": 3}[args.store])
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
