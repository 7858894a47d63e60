"""Pins the CPU oracle to the reference: every golden case, outputs and gradients.

The golden vectors come from the reference's own ``native`` backend
(tests/golden/make_golden.py). CPU-only.
"""
import numpy as np
import pytest
import torch

from oracle import fp64_backward, fp64_forward, native_forward_backward
from tests._util import assert_ulp, rel_err, ulp_diff

pytestmark = pytest.mark.filterwarnings("ignore::UserWarning")


def _dense(case):
    """Golden tensors as dense [B,H,N,D] float64 numpy plus sin/cos [B|1,1,N,D/2]."""
    q, k = case.q.double(), case.k.double()
    gq, gk = case.gq.double(), case.gk.double()
    sin, cos = case.sin.double(), case.cos.double()
    if case.packed:
        q, k, gq, gk = (x.transpose(0, 1)[None] for x in (q, k, gq, gk))
        sin, cos = sin[None, None], cos[None, None]
    elif sin.ndim == 2:
        sin, cos = sin[None, None], cos[None, None]
    else:
        sin, cos = sin[:, None], cos[:, None]
    return [x.numpy() for x in (q, k, gq, gk, sin, cos)]


def _to_case_layout(case, x):
    x = torch.from_numpy(np.ascontiguousarray(x))
    return x[0].transpose(0, 1) if case.packed else x


def test_golden_file_has_all_cases(golden):
    assert len(golden) >= 18
    assert {"c1_slice", "c2_slice", "c3_slice", "c4_slice"} <= set(golden)


@pytest.mark.parametrize("name", sorted(__import__("tests.golden", fromlist=["x"]).load_golden()))
def test_native_restatement_matches_reference(golden, name):
    case = golden[name]
    torch.set_num_threads(1)
    args = case.args("cpu")
    outs, grads = native_forward_backward(*args, case.gq, case.gk, eps=case.eps)
    # Same ops in the same order as the reference: at most 1 ulp (the CPU's
    # reduction schedule is the only source of difference across machines).
    d_q = assert_ulp(outs[0], case.q_out, 1, "q_out")
    d_k = assert_ulp(outs[1], case.k_out, 1, "k_out")
    assert float((d_q == 0).float().mean()) > 0.999 and float((d_k == 0).float().mean()) > 0.999
    tol = dict(atol=1e-6, rtol=1e-5) if case.dtype == torch.float32 else dict(atol=0, rtol=0.0079)
    torch.testing.assert_close(grads[0], case.dq, **tol)
    torch.testing.assert_close(grads[1], case.dk, **tol)
    assert rel_err(grads[2], case.dw) < 1e-5
    assert rel_err(grads[3], case.ds) < 1e-5


@pytest.mark.parametrize("name", sorted(__import__("tests.golden", fromlist=["x"]).load_golden()))
def test_fp64_oracle_matches_reference(golden, name):
    case = golden[name]
    q, k, gq, gk, sin, cos = _dense(case)
    w = case.w.double().numpy()
    s = case.s.double().numpy().reshape(-1)
    oq, ok = fp64_forward(q, k, w, s, sin, cos, eps=case.eps)
    for got, ref, nm in ((oq, case.q_out, "q_out"), (ok, case.k_out, "k_out")):
        got = _to_case_layout(case, got)
        if case.dtype == torch.float32:
            torch.testing.assert_close(got.float(), ref, rtol=1e-5, atol=1e-5)
            continue
        # The reference rounds FP32 intermediates; exact FP64 may land 1 ulp away.
        d = ulp_diff(got.to(case.dtype), ref)
        assert int(d.max()) <= 1, nm
        assert float((d == 0).float().mean()) > 0.97, nm
    dq, dk, dw, ds = fp64_backward(q, k, w, s, sin, cos, gq, gk, eps=case.eps)
    for got, ref in ((dq, case.dq), (dk, case.dk)):
        got = _to_case_layout(case, got)
        scale = ref.double().abs().max().clamp_min(1e-6)
        assert float((got - ref.double()).abs().max() / scale) < 2e-2
    assert rel_err(torch.from_numpy(dw), case.dw) < 1e-3
    assert rel_err(torch.from_numpy(ds), case.ds) < 1e-3
