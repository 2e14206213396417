"""Gated-scan backward on the GPU against the reference's gradients (golden
vectors from autograd through affine_scan.py) and the oracle's backward."""
import numpy as np
import pytest
import torch

from oracle import scan_oracle as O
from tests.golden.make_golden import headed_inputs
from tests.helpers import as64, headed_bf16, rel_max_err

pytestmark = pytest.mark.gpu
TOL_F32 = 1e-4
TOL_BF16 = 2e-2


@pytest.fixture(scope="module")
def mg():
    import mogt_b200
    return mogt_b200


def _grads(m, q, k, v, f, g, S0=None):
    ins = [t.cuda().requires_grad_(True) for t in (q, k, v, f)]
    s0 = None if S0 is None else S0.cuda().requires_grad_(True)
    o = m.gated_scan(*ins, initial_state=s0)
    (o.float() * g.cuda()).sum().backward()
    out = [t.grad for t in ins]
    if s0 is not None:
        out.append(s0.grad)
    return out


def test_config1_fp32_grads_match_reference(mg, golden):
    d = golden("config1_fp32")
    q, k, v, f, g = headed_inputs(2, 4, 512, 32, 32, torch.float32)
    dq, dk, dv, df = _grads(mg, q, k, v, f, g)
    for got, key in [(dq, "dq"), (dk, "dk"), (dv, "dv"), (df, "df")]:
        assert rel_max_err(got.cpu().numpy(), d[key]) <= TOL_F32, key


def test_small_fp64_golden_in_fp32(mg, golden):
    d = golden("headed_small_fp64")
    ts = [torch.from_numpy(d[x]).float() for x in ("q", "k", "v", "f", "g")]
    dq, dk, dv, df = _grads(mg, *ts)
    for got, key in [(dq, "dq"), (dk, "dk"), (dv, "dv"), (df, "df")]:
        assert rel_max_err(got.cpu().numpy(), d[key]) <= TOL_F32, key


@pytest.mark.parametrize("T", [1, 63, 64, 65, 300])
def test_fp32_ragged_lengths_vs_oracle(mg, T):
    q, k, v, f, g = headed_inputs(1, 2, T, 16, 24, torch.float32, seed=T)
    dq, dk, dv, df = _grads(mg, q, k, v, f, g)
    ref = O.gated_scan_backward(*as64(q, k, v, f, g))
    for got, r in zip((dq, dk, dv, df), ref):
        assert rel_max_err(got.cpu().numpy(), r) <= TOL_F32


def test_initial_state_gradient(mg):
    """dS0 = f_0 G_0, checked against float64 autograd through the recurrence."""
    q, k, v, f, g = headed_inputs(1, 2, 50, 8, 8, torch.float32, seed=3)
    S0 = torch.randn(1, 2, 8, 8)
    dq, dk, dv, df, dS0 = _grads(mg, q, k, v, f, g, S0)
    ins = [t.double().requires_grad_(True) for t in (q, k, v, f, S0)]
    qd, kd, vd, fd, Sd = ins
    S, outs = Sd, []
    for t in range(50):
        ft = fd[:, :, t, None, None]
        S = ft * S + (1 - ft) * kd[:, :, t, :, None] * vd[:, :, t, None, :]
        outs.append(torch.einsum("bhkv,bhk->bhv", S, qd[:, :, t]))
    o = torch.stack(outs, 2)
    (o * g.double()).sum().backward()
    for got, ref in zip((dq, dk, dv, df, dS0), ins):
        assert rel_max_err(got.cpu().numpy(), ref.grad.numpy()) <= TOL_F32


def test_bf16_inputs_backward(mg):
    q, k, v, f = headed_bf16(1, 2, 200, seed=9)
    g = torch.randn(1, 2, 200, 64)
    dq, dk, dv, df = _grads(mg, q, k, v, f, g)
    assert dq.dtype == torch.bfloat16 and df.dtype == torch.float32
    ref = O.gated_scan_backward(*as64(q, k, v, f, g))
    for got, r in zip((dq, dk, dv, df), ref):
        assert rel_max_err(got.float().cpu().numpy(), r) <= TOL_BF16
