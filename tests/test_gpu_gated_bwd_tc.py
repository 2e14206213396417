"""Tensor-core (bf16, 64x64) gated-scan backward: the reverse-time chunked
kernel against the oracle's backward on the same bf16-rounded inputs, for
ragged lengths, multi-stripe look-back, gates at 0 / 1 / tiny values, an
initial state, and at the config-2 size against the exact fp32 sequential
kernel."""
import numpy as np
import pytest
import torch

from oracle import scan_oracle as O
from tests.helpers import as64, headed_bf16, rel_max_err

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2


@pytest.fixture(scope="module")
def mg():
    import mogt_b200
    return mogt_b200


def _tc_grads(m, q, k, v, f, g, S0=None):
    """Forward with saved chunk states, then the tensor-core backward."""
    qc, kc, vc, fc = (t.cuda() for t in (q, k, v, f))
    s0 = None if S0 is None else S0.cuda()
    _, _, _, cs = m.ops.gated_scan_fwd(qc, kc, vc, fc, initial_state=s0, save_states=True)
    return m.ops.gated_scan_bwd(qc, kc, vc, fc, g.cuda().bfloat16(), chunk_states=cs,
                                want_dS0=S0 is not None)


def _oracle(q, k, v, f, g):
    return O.gated_scan_backward(*as64(q, k, v, f, g.bfloat16()))


@pytest.mark.parametrize("T", [1, 37, 64, 65, 200, 1000])
def test_ragged_lengths_vs_oracle(mg, T):
    q, k, v, f = headed_bf16(1, 3, T, seed=100 + T)
    g = torch.randn(1, 3, T, 64, generator=torch.Generator().manual_seed(T))
    dq, dk, dv, df, _ = _tc_grads(mg, q, k, v, f, g)
    assert dq.dtype == torch.bfloat16 and df.dtype == torch.float32
    ref = _oracle(q, k, v, f, g)
    for name, got, r in zip(("dq", "dk", "dv", "df"), (dq, dk, dv, df), ref):
        assert rel_max_err(got.float().cpu().numpy(), r) <= TOL_BF16, name


def test_many_stripes_lookback_vs_oracle(mg):
    """T = 2048, BH = 2: one chunk per stripe, 32-deep look-back chains."""
    q, k, v, f = headed_bf16(1, 2, 2048, seed=7)
    g = torch.randn(1, 2, 2048, 64, generator=torch.Generator().manual_seed(1))
    dq, dk, dv, df, _ = _tc_grads(mg, q, k, v, f, g)
    ref = _oracle(q, k, v, f, g)
    for name, got, r in zip(("dq", "dk", "dv", "df"), (dq, dk, dv, df), ref):
        assert rel_max_err(got.float().cpu().numpy(), r) <= TOL_BF16, name


@pytest.mark.parametrize("mode", ["mixed", "zeros", "ones"])
def test_extreme_gates_vs_oracle(mg, mode):
    """Gates of exactly 0 (full reset), 1 (no write) and 1e-3: decays far
    below 2^-100 inside a chunk, which the per-element decay form handles."""
    q, k, v, f = headed_bf16(1, 2, 700, seed=5, f_mode=mode)
    g = torch.randn(1, 2, 700, 64, generator=torch.Generator().manual_seed(2))
    dq, dk, dv, df, _ = _tc_grads(mg, q, k, v, f, g)
    ref = _oracle(q, k, v, f, g)
    for name, got, r in zip(("dq", "dk", "dv", "df"), (dq, dk, dv, df), ref):
        r = np.asarray(r)
        if np.abs(r).max() == 0:
            assert float(got.float().abs().max()) == 0.0, name
        else:
            assert rel_max_err(got.float().cpu().numpy(), r) <= TOL_BF16, name


def test_initial_state_and_its_gradient(mg):
    """With S0, against float64 autograd through the recurrence."""
    T = 300
    q, k, v, f = headed_bf16(1, 2, T, seed=21)
    g = torch.randn(1, 2, T, 64, generator=torch.Generator().manual_seed(3))
    S0 = torch.randn(1, 2, 64, 64, generator=torch.Generator().manual_seed(4))
    dq, dk, dv, df, dS0 = _tc_grads(mg, q, k, v, f, g, S0)
    ins = [t.double().requires_grad_(True) for t in (q, k, v, f, S0)]
    qd, kd, vd, fd, Sd = ins
    S, outs = Sd, []
    for t in range(T):
        ft = fd[:, :, t, None, None]
        S = ft * S + (1 - ft) * kd[:, :, t, :, None] * vd[:, :, t, None, :]
        outs.append(torch.einsum("bhkv,bhk->bhv", S, qd[:, :, t]))
    (torch.stack(outs, 2) * g.bfloat16().double()).sum().backward()
    for name, got, ref in zip(("dq", "dk", "dv", "df", "dS0"), (dq, dk, dv, df, dS0), ins):
        assert rel_max_err(got.float().cpu().numpy(), ref.grad.numpy()) <= TOL_BF16, name


def test_autograd_uses_tensor_core_path(mg):
    q, k, v, f = headed_bf16(1, 2, 333, seed=8)
    g = torch.randn(1, 2, 333, 64, generator=torch.Generator().manual_seed(5))
    ins = [t.cuda().requires_grad_(True) for t in (q, k, v, f)]
    o = mg.gated_scan(*ins)
    (o.float() * g.cuda()).sum().backward()
    ref = _oracle(q, k, v, f, g)
    for name, t, r in zip(("dq", "dk", "dv", "df"), ins, ref):
        assert rel_max_err(t.grad.float().cpu().numpy(), r) <= TOL_BF16, name


def test_config2_size_vs_fp32_sequential(mg):
    """B=1, H=12, T=32768: against the exact fp32 sequential backward on the
    same (bf16-rounded) inputs."""
    B, H, T = 1, 12, 32768
    q, k, v, f = (t.cuda() for t in headed_bf16(B, H, T, seed=2))
    g = torch.randn(B, H, T, 64, device="cuda").bfloat16()
    _, _, _, cs = mg.ops.gated_scan_fwd(q, k, v, f, save_states=True)
    got = mg.ops.gated_scan_bwd(q, k, v, f, g, chunk_states=cs)
    ref = mg.ops.gated_scan_bwd(q.float(), k.float(), v.float(), f, g.float())
    for name, a, r in zip(("dq", "dk", "dv", "df"), got[:4], ref[:4]):
        err = float((a.float() - r).abs().max() / r.abs().max())
        assert err <= TOL_BF16, (name, err)
    from mogt_b200 import _native as N
    assert all(e == 0 for e in N.workspace_errors())
