"""Parity at the BASELINE sizes against the oracle, over every head and every
step (not samples, and not the CUDA path against itself).

* config 2 forward: B=1, H=12, dk=dv=64, T in {8192, 16384, 32768}, bf16
  inputs, fp32 output, against O.gated_scan in float64;
* config 2 backward: T=8192, all 12 heads, against O.gated_scan_backward;
* config 3 forward: B=2, H=8, T=8192, d=64 Cayley transitions, against the
  streaming float64 oracle (affine_scan.py:14-62 stepped per t).

Tolerances (north star): bf16 inputs with fp32 accumulation <= 2e-2 relative
(max-abs error over max-abs reference); fp32 arithmetic <= 1e-4.  Each test
also bounds the relative Frobenius error, and appends its figures to the
JSON-lines file named by MOGT_PARITY_LOG when that variable is set.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import scan_oracle as O
from tests.helpers import as64, headed_bf16, rel_fro_err, rel_max_err

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2
TOL_F32 = 1e-4


def _log(**rec):
    path = os.environ.get("MOGT_PARITY_LOG")
    if path:
        with open(path, "a") as fh:
            fh.write(json.dumps(rec) + "\n")


@pytest.mark.parametrize("T", [8192, 16384, 32768])
def test_config2_forward_all_heads_full_length(T):
    import mogt_b200
    q, k, v, f = headed_bf16(1, 12, T, seed=100 + T // 8192)
    o = mogt_b200.gated_scan(q.cuda(), k.cuda(), v.cuda(), f.cuda(), output_dtype=torch.float32)
    o = o.cpu().numpy()
    ref = O.gated_scan(*as64(q, k, v, f))
    e_max, e_fro = rel_max_err(o, ref), rel_fro_err(o, ref)
    # the last 2048 steps separately: an error in a late stripe or look-back
    # would show there first
    e_tail = rel_max_err(o[:, :, -2048:], ref[:, :, -2048:])
    _log(test="config2_fwd", T=T, heads=12, rel_max=e_max, rel_fro=e_fro, rel_max_tail=e_tail)
    assert e_max <= TOL_BF16 and e_tail <= TOL_BF16
    assert e_fro <= 5e-3


def test_config2_bf16_output_full_length():
    """The bench's output dtype (bf16) at T = 32768: the extra rounding of o
    stays inside the bf16 bar."""
    import mogt_b200
    T = 32768
    q, k, v, f = headed_bf16(1, 12, T, seed=104)
    o = mogt_b200.gated_scan(q.cuda(), k.cuda(), v.cuda(), f.cuda()).float().cpu().numpy()
    ref = O.gated_scan(*as64(q, k, v, f))
    e_max, e_fro = rel_max_err(o, ref), rel_fro_err(o, ref)
    _log(test="config2_fwd_bf16_out", T=T, heads=12, rel_max=e_max, rel_fro=e_fro)
    assert e_max <= TOL_BF16 and e_fro <= 1e-2


def test_config2_backward_all_heads_T8192():
    import mogt_b200
    T = 8192
    q, k, v, f = headed_bf16(1, 12, T, seed=208)
    g = torch.randn(1, 12, T, 64, generator=torch.Generator().manual_seed(209)).bfloat16()
    qc, kc, vc, fc = (t.cuda() for t in (q, k, v, f))
    _, _, _, cs = mogt_b200.ops.gated_scan_fwd(qc, kc, vc, fc, save_states=True)
    dq, dk, dv, df, _ = mogt_b200.ops.gated_scan_bwd(qc, kc, vc, fc, g.cuda(), chunk_states=cs)
    refs = O.gated_scan_backward(*as64(q, k, v, f, g))
    rec = {}
    for name, got, ref in zip(("dq", "dk", "dv", "df"), (dq, dk, dv, df), refs):
        got = got.float().cpu().numpy()
        rec[name] = (rel_max_err(got, ref), rel_fro_err(got, ref))
    _log(test="config2_bwd", T=T, heads=12, **{k: {"rel_max": a, "rel_fro": b} for k, (a, b) in rec.items()})
    for name, (e_max, e_fro) in rec.items():
        assert e_max <= TOL_BF16, (name, e_max)
        assert e_fro <= 1e-2, (name, e_fro)


def _cayley_gpu(B, H, T, d, seed):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(seed)
    A = torch.empty(B, H, T, d, d, dtype=torch.float32, device=dev)
    I = torch.eye(d, dtype=torch.float64, device=dev)
    for t0 in range(0, T, 1024):
        M = torch.randn(B, H, min(1024, T - t0), d, d, generator=g, dtype=torch.float64, device=dev)
        W = 0.05 * (M - M.transpose(-1, -2))
        A[:, :, t0:t0 + M.shape[2]] = torch.linalg.solve(I - W, I + W).float()
    return A


def test_config3_forward_all_heads_full_length():
    """Norm-preserving transitions never forget round-off, so this is the
    check of the 3xTF32 scheme's accumulated error over all 8192 steps."""
    import mogt_b200
    B, H, T, d = 2, 8, 8192, 64
    A = _cayley_gpu(B, H, T, d, seed=31)
    gen = torch.Generator().manual_seed(32)
    q, k, v = (torch.randn(B, H, T, d, generator=gen).bfloat16() for _ in range(3))
    f = torch.sigmoid(torch.randn(B, H, T, generator=gen) + 2.0)
    o, S = mogt_b200.ops.matrix_scan_fwd(A, q.cuda(), k.cuda(), v.cuda(), f.cuda(),
                                         output_dtype=torch.float32, want_final=True)
    o = o.cpu().numpy()
    S = S.cpu().numpy()
    A_h = A.cpu().numpy()
    del A
    torch.cuda.empty_cache()
    ref, Sref = O.matrix_scan_stream(A_h, *as64(q, k, v, f), return_final=True)
    e_max, e_fro = rel_max_err(o, ref), rel_fro_err(o, ref)
    e_tail = rel_max_err(o[:, :, -512:], ref[:, :, -512:])
    e_S = rel_max_err(S, Sref)
    _log(test="config3_fwd", T=T, heads=B * H, rel_max=e_max, rel_fro=e_fro, rel_max_tail=e_tail,
         rel_max_final_state=e_S)
    assert e_max <= TOL_F32 and e_tail <= TOL_F32 and e_S <= TOL_F32
    assert e_fro <= TOL_F32
