"""Pins the inverse-formulation oracle to the reference-generated golden vectors (CPU).

The inverse forward is the ``native`` forward plus r per row, so its outputs
must equal the golden outputs. The inverse backward rebuilds the normalised
rows from the outputs; fed the golden outputs it must reproduce the golden
(autograd) gradients up to the rounding of those outputs: FP32 cases within
FP32 rounding, FP16/BF16 cases within the output dtype's rounding.
"""
import pytest
import torch

from oracle import fp64_forward, inverse_backward, inverse_forward
from tests._util import assert_ulp, rel_err

CASES = sorted(__import__("tests.golden", fromlist=["x"]).load_golden())
# Relative L2 bounds on (dq, dk, dw, ds) per activation dtype: the error of
# rebuilding the rows from outputs rounded to that dtype (measured: FP32
# <= 4e-7, FP16 <= 3e-4, BF16 <= 3.5e-3).
BOUNDS = {torch.float32: 2e-6, torch.float16: 1e-3, torch.bfloat16: 6e-3}


def _dense(case):
    """(q, k, w, s, sin, cos, gq, gk) as 4-D [B,H,N,D] views, sin/cos [B|1,1,N,D/2]."""
    q, k, w, s, sin, cos = case.args("cpu")
    gq, gk = case.gq, case.gk
    if case.packed:
        q, k, gq, gk = (x.transpose(0, 1)[None] for x in (q, k, gq, gk))
        sin, cos = sin[None, None], cos[None, None]
    elif sin.ndim == 2:
        sin, cos = sin[None, None], cos[None, None]
    elif sin.ndim == 3:
        sin, cos = sin[:, None], cos[:, None]
    return q, k, w, s, sin, cos, gq, gk


def _golden4(case, x):
    return x.transpose(0, 1)[None] if case.packed else x


@pytest.mark.parametrize("name", CASES)
def test_inverse_forward_outputs_and_statistic(golden, name):
    case = golden[name]
    torch.set_num_threads(1)
    q, k, w, s, sin, cos, _, _ = _dense(case)
    q_out, k_out, rms_q, rms_k = inverse_forward(q, k, w, s, sin, cos, eps=case.eps)
    assert_ulp(q_out.contiguous(), _golden4(case, case.q_out).contiguous(), 1, "q_out")
    assert_ulp(k_out.contiguous(), _golden4(case, case.k_out).contiguous(), 1, "k_out")
    assert rms_q.shape == (*q.shape[:3], 1) and rms_q.dtype == torch.float32
    for x, r in ((q, rms_q), (k, rms_k)):
        exact = 1.0 / torch.sqrt(x.double().square().mean(-1, keepdim=True) + case.eps)
        torch.testing.assert_close(r.double(), exact, rtol=1e-6, atol=0)


@pytest.mark.parametrize("name", CASES)
def test_inverse_backward_reproduces_reference_gradients(golden, name):
    case = golden[name]
    torch.set_num_threads(1)
    q, k, w, s, sin, cos, gq, gk = _dense(case)
    _, _, rms_q, rms_k = inverse_forward(q, k, w, s, sin, cos, eps=case.eps)
    dq, dk, dw, ds = inverse_backward(_golden4(case, case.q_out), _golden4(case, case.k_out), w, s,
                                      sin, cos, gq, gk, rms_q, rms_k)
    bound = BOUNDS[case.dtype]
    assert dq.dtype == case.dtype and dq.shape == q.shape
    assert rel_err(dq.float(), _golden4(case, case.dq).float()) < bound
    assert rel_err(dk.float(), _golden4(case, case.dk).float()) < bound
    assert rel_err(dw, case.dw) < bound
    assert rel_err(ds, case.ds) < bound


def test_inverse_backward_planted_error_is_caught(golden):
    """A wrong saved statistic (r of the wrong tensor) must fail the bar above."""
    case = golden["ref_fp32_t32"]
    q, k, w, s, sin, cos, gq, gk = _dense(case)
    _, _, rms_q, rms_k = inverse_forward(q, k, w, s, sin, cos, eps=case.eps)
    dq, *_ = inverse_backward(_golden4(case, case.q_out), _golden4(case, case.k_out), w, s, sin, cos,
                              gq, gk, rms_k, rms_q)
    assert rel_err(dq.float(), _golden4(case, case.dq).float()) > 100 * BOUNDS[torch.float32]


def test_inverse_forward_matches_fp64_statistic():
    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 3, 5, 64, generator=g)
    k = torch.randn(2, 3, 5, 64, generator=g)
    w = 1 + 0.02 * torch.randn(2, 1, 64, generator=g)
    s = 0.1 * torch.randn(3, 1, 1, generator=g)
    ang = torch.rand(1, 1, 5, 32, generator=g)
    _, _, rq, _ = inverse_forward(q, k, w, s, ang.sin(), ang.cos(), eps=0.1)
    exact = 1.0 / torch.sqrt(q.double().square().mean(-1, keepdim=True) + 0.1)
    torch.testing.assert_close(rq.double(), exact, rtol=1e-6, atol=0)
    # The outputs are those of the independent FP64 oracle to FP32 rounding.
    oq, _ = fp64_forward(q.double().numpy(), k.double().numpy(), w.double().numpy(),
                         s.double().numpy().reshape(-1), ang.sin().double().numpy(),
                         ang.cos().double().numpy(), eps=0.1)
    qo, *_ = inverse_forward(q, k, w, s, ang.sin(), ang.cos(), eps=0.1)
    torch.testing.assert_close(qo.double(), torch.from_numpy(oq), rtol=1e-5, atol=1e-5)
