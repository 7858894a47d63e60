"""Generates tests/golden/prologue_golden.npz from the reference implementation.

Run in a container that has the reference checkout (it is NOT available on the
GPU box, which only reads the committed .npz):

    python tests/golden/make_golden.py --reference /path/to/flash_attn_prologue_checkout

For each case it builds seeded inputs (numpy PCG64, platform independent),
calls the reference's public ``qknorm_rope_scale(..., backend="native")`` on
CPU (flash_attn_prologue/functional.py:14-94) and backpropagates seeded
upstream gradients with torch.autograd, then stores inputs, outputs and the
four gradients. BF16/FP16 tensors are stored as their raw 16-bit patterns.
Shapes follow the reference's own tests (tests/test_frontend_api.py:35-47,
76-86, 225-234) and token/position slices of the benchmark configurations.
"""
import argparse
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "prologue_golden.npz"

DT = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}


def rope_tables(positions, d, theta):
    inv_freq = 1.0 / (theta ** (np.arange(0, d, 2, dtype=np.float64) / d))
    ang = np.outer(np.asarray(positions, dtype=np.float64), inv_freq).astype(np.float32)
    return np.sin(ang), np.cos(ang)


def case_specs():
    """(name, spec) pairs; spec fully determines the inputs."""
    specs = []
    # Reference frontend test shapes: H=4, w=1+0.2N, s=0.2N-log(d)/2, random angles.
    for t, d, packed, nc in [(1, 32, True, False), (63, 32, True, False), (64, 32, True, False),
                             (65, 32, True, True), (95, 64, False, False), (96, 64, True, False),
                             (127, 32, False, True), (128, 64, True, False), (129, 32, True, False),
                             (17, 32, False, False)]:
        specs.append((f"ref_t{t}_d{d}_{'packed' if packed else 'dense'}{'_nc' if nc else ''}",
                      dict(kind="ref", t=t, d=d, h=4, packed=packed, noncontig=nc, dtype="bf16",
                           eps=1e-5, seed=832 + t + d)))
    specs.append(("ref_fp16_t32", dict(kind="ref", t=32, d=32, h=4, packed=True, noncontig=False,
                                       dtype="fp16", eps=1e-5, seed=7)))
    specs.append(("ref_fp32_t32", dict(kind="ref", t=32, d=32, h=4, packed=True, noncontig=False,
                                       dtype="fp32", eps=1e-5, seed=8)))
    specs.append(("ref_fp32_t17_eps0.1", dict(kind="ref", t=17, d=32, h=4, packed=True,
                                              noncontig=False, dtype="fp32", eps=0.1, seed=9)))
    # Slices of the benchmark configurations (rows are independent, so a token
    # slice exercises exactly the arithmetic of the full run).
    specs.append(("c1_slice", dict(kind="c1", t=256, d=32, h=4, theta=10000.0, seed=1)))
    specs.append(("c2_slice", dict(kind="c2", t=64, d=64, h=16, theta=10000.0, seed=2)))
    specs.append(("c3_slice", dict(kind="c3", b=1, s=64, d=128, h=4, theta=500000.0, seed=3)))
    specs.append(("c4_slice", dict(kind="c4", t=64, d=64, h=8, theta=10000.0, seed=4)))
    specs.append(("d256_packed", dict(kind="ref", t=16, d=256, h=2, packed=True, noncontig=False,
                                      dtype="bf16", eps=1e-5, seed=5)))
    return specs


def make_inputs(spec):
    """Returns dict of numpy arrays (float32 for activations before the cast)."""
    rng = np.random.Generator(np.random.PCG64(spec["seed"]))
    kind, d, h = spec["kind"], spec["d"], spec["h"]
    if kind == "ref":
        t = spec["t"]
        shape = (t, h, d) if spec["packed"] else (2, h, t, d)
        q = rng.standard_normal(shape, dtype=np.float32)
        k = rng.standard_normal(shape, dtype=np.float32)
        w = (1 + rng.standard_normal((2, 1, d), dtype=np.float32) * 0.2).astype(np.float32)
        s = (rng.standard_normal((h, 1, 1), dtype=np.float32) * 0.2 - math.log(d) / 2).astype(np.float32)
        ang = rng.standard_normal((t, d // 2) if spec["packed"] else (2, t, d // 2), dtype=np.float32)
        sin, cos = np.sin(ang), np.cos(ang)
        layout = "packed" if spec["packed"] else "dense"
    elif kind == "c1":
        t = spec["t"]
        q = rng.standard_normal((t, h, d), dtype=np.float32)
        k = rng.standard_normal((t, h, d), dtype=np.float32)
        w = (1 + rng.standard_normal((2, 1, d), dtype=np.float32) * 0.02).astype(np.float32)
        s = np.zeros((h, 1, 1), dtype=np.float32)
        sin, cos = rope_tables(np.arange(t), d, spec["theta"])
        layout = "packed"
    elif kind == "c2":
        t = spec["t"]
        buf = rng.standard_normal((t, 3, h, d), dtype=np.float32)
        q, k = buf[:, 0], buf[:, 1]
        w = (1 + rng.standard_normal((2, 1, d), dtype=np.float32) * 0.02).astype(np.float32)
        s = (rng.standard_normal((h, 1, 1), dtype=np.float32) * 0.1).astype(np.float32)
        sin, cos = rope_tables((np.arange(t) * 37) % 4096, d, spec["theta"])
        layout = "qkv_packed"
    elif kind == "c3":
        b, n = spec["b"], spec["s"]
        q = rng.standard_normal((b, h, n, d), dtype=np.float32)
        k = rng.standard_normal((b, h, n, d), dtype=np.float32)
        w = (1 + rng.standard_normal((2, 1, d), dtype=np.float32) * 0.02).astype(np.float32)
        s = np.full((h, 1, 1), math.log(1 / math.sqrt(d)), dtype=np.float32)
        sin, cos = rope_tables(np.arange(n), d, spec["theta"])
        layout = "dense"
    elif kind == "c4":
        t = spec["t"]
        q = rng.standard_normal((t, h, d), dtype=np.float32)
        k = rng.standard_normal((t, h, d), dtype=np.float32)
        w = (1 + rng.standard_normal((2, 1, d), dtype=np.float32) * 0.02).astype(np.float32)
        s = (rng.standard_normal((h, 1, 1), dtype=np.float32) * 0.1).astype(np.float32)
        sin, cos = rope_tables(np.arange(t), d, spec["theta"])
        layout = "packed"
    else:
        raise ValueError(kind)
    gq = rng.standard_normal(q.shape, dtype=np.float32)
    gk = rng.standard_normal(k.shape, dtype=np.float32)
    return dict(q=np.ascontiguousarray(q), k=np.ascontiguousarray(k), w=w, s=s,
                sin=np.ascontiguousarray(sin), cos=np.ascontiguousarray(cos),
                gq=gq, gk=gk, layout=layout)


def to_bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float32:
        return t.detach().contiguous().numpy()
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def run_reference(qknorm_rope_scale, inp, dtype, eps):
    tq = torch.from_numpy(inp["q"]).to(dtype).requires_grad_()
    tk = torch.from_numpy(inp["k"]).to(dtype).requires_grad_()
    tw = torch.from_numpy(inp["w"]).requires_grad_()
    ts = torch.from_numpy(inp["s"]).requires_grad_()
    sin, cos = torch.from_numpy(inp["sin"]), torch.from_numpy(inp["cos"])
    out = qknorm_rope_scale(tq, tk, tw, ts, sin, cos, eps, backend="native")
    gq = torch.from_numpy(inp["gq"]).to(dtype)
    gk = torch.from_numpy(inp["gk"]).to(dtype)
    grads = torch.autograd.grad(out, (tq, tk, tw, ts), (gq, gk))
    return tq, tk, gq, gk, out, grads


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True,
                    help="directory that contains the reference flash_attn_prologue package")
    ap.add_argument("--out", default=str(OUT))
    args = ap.parse_args(argv)
    sys.path.insert(0, args.reference)
    from flash_attn_prologue.functional import qknorm_rope_scale  # the reference itself

    torch.set_num_threads(1)  # one reduction schedule for the CPU mean
    arrays, meta = {}, {}
    for name, spec in case_specs():
        inp = make_inputs(spec)
        dtype = DT[spec.get("dtype", "bf16")]
        eps = spec.get("eps", 1e-5)
        tq, tk, gq, gk, out, grads = run_reference(qknorm_rope_scale, inp, dtype, eps)
        rec = dict(q=to_bits(tq), k=to_bits(tk), w=inp["w"], s=inp["s"], sin=inp["sin"],
                   cos=inp["cos"], gq=to_bits(gq), gk=to_bits(gk), q_out=to_bits(out[0]),
                   k_out=to_bits(out[1]), dq=to_bits(grads[0]), dk=to_bits(grads[1]),
                   dw=grads[2].numpy(), ds=grads[3].numpy())
        for key, val in rec.items():
            arrays[f"{name}/{key}"] = val
        meta[name] = dict(spec, layout=inp["layout"], dtype=spec.get("dtype", "bf16"), eps=eps)
    arrays["__meta__"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **arrays)
    print(f"wrote {args.out}: {len(meta)} cases, {Path(args.out).stat().st_size} bytes")


if __name__ == "__main__":
    main()
