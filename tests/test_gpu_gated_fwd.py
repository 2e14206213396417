"""Gated (headed) scan forward on the GPU vs the oracle.

Tolerances (north star): fp32 inputs <= 1e-4 relative; bf16 inputs with fp32
accumulation <= 2e-2 relative (max-abs error over max-abs reference)."""
import numpy as np
import pytest
import torch

from oracle import scan_oracle as O
from tests.golden.make_golden import headed_inputs
from tests.helpers import as64, headed_bf16, rel_fro_err, rel_max_err

pytestmark = pytest.mark.gpu
TOL_F32 = 1e-4
TOL_BF16 = 2e-2


@pytest.fixture(scope="module")
def mg():
    import mogt_b200
    from mogt_b200 import _native
    assert torch.cuda.is_available()
    return mogt_b200, _native


def test_config1_fp32_golden(mg, golden):
    m, _ = mg
    d = golden("config1_fp32")
    q, k, v, f, g = headed_inputs(2, 4, 512, 32, 32, torch.float32)
    o = m.gated_scan(q.cuda(), k.cuda(), v.cuda(), f.cuda())
    assert o.dtype == torch.float32
    assert rel_max_err(o.cpu().numpy(), d["o"]) <= TOL_F32


@pytest.mark.parametrize("T", [1, 17, 64, 255, 256, 257, 700, 2048])
def test_bf16_matches_oracle(mg, T):
    m, N = mg
    q, k, v, f = headed_bf16(1, 3, T, seed=T)
    o = m.gated_scan(q.cuda(), k.cuda(), v.cuda(), f.cuda())
    assert o.dtype == torch.bfloat16 and o.shape == (1, 3, T, 64)
    ref = O.gated_scan(*as64(q, k, v, f))
    assert rel_max_err(o.float().cpu().numpy(), ref) <= TOL_BF16
    assert rel_fro_err(o.float().cpu().numpy(), ref) <= 5e-3
    assert all(e == 0 for e in N.workspace_errors())


@pytest.mark.parametrize("mode", ["ones", "zeros", "mixed"])
def test_bf16_gate_edge_cases(mg, mode):
    m, _ = mg
    q, k, v, f = headed_bf16(2, 2, 600, seed=5, f_mode=mode)
    S0 = torch.randn(2, 2, 64, 64)
    o, S_fin, dec, _ = m.ops.gated_scan_fwd(q.cuda(), k.cuda(), v.cuda(), f.cuda(),
                                            initial_state=S0.cuda(), output_dtype=torch.float32,
                                            want_final=True)
    ref, Sref = O.gated_scan(*as64(q, k, v, f), S0=S0.double().numpy(), return_final=True)
    assert rel_max_err(o.cpu().numpy(), ref) <= TOL_BF16
    assert rel_max_err(S_fin.cpu().numpy(), Sref) <= TOL_BF16
    dref = np.prod(f.double().numpy(), axis=-1)
    assert np.allclose(dec.cpu().numpy(), dref, rtol=1e-3, atol=1e-30)


def test_fp32_initial_and_final_state(mg):
    m, _ = mg
    q, k, v, f, _ = headed_inputs(1, 2, 300, 48, 40, torch.float32)
    S0 = torch.randn(1, 2, 48, 40)
    o, S_fin, dec, _ = m.ops.gated_scan_fwd(q.cuda(), k.cuda(), v.cuda(), f.cuda(),
                                            initial_state=S0.cuda(), want_final=True)
    ref, Sref = O.gated_scan(*as64(q, k, v, f), S0=S0.double().numpy(), return_final=True)
    assert rel_max_err(o.cpu().numpy(), ref) <= TOL_F32
    assert rel_max_err(S_fin.cpu().numpy(), Sref) <= TOL_F32


def test_chunk_states_and_state_only_mode(mg):
    m, _ = mg
    T = 1100
    q, k, v, f = headed_bf16(1, 2, T, seed=11)
    o, S_fin, dec, seg = m.ops.gated_scan_fwd(q.cuda(), k.cuda(), v.cuda(), f.cuda(),
                                              want_final=True, save_states=True)
    assert seg.shape == (1, 2, 18, 64, 64) and seg.dtype == torch.bfloat16
    # state entering chunk c is S_{64 c - 1} (bf16-rounded)
    kk, vv, ff = as64(k, v, f)
    S = np.zeros((2, 64, 64))
    assert float(seg[0, :, 0].abs().max()) == 0.0
    for t in range(T):
        if t % 64 == 0 and t > 0:
            assert rel_max_err(seg[0, :, t // 64].float().cpu().numpy(), S) <= TOL_BF16
        S = ff[0, :, t, None, None] * S + (1 - ff[0, :, t, None, None]) * kk[0, :, t, :, None] * vv[0, :, t, None, :]
    assert rel_max_err(S_fin[0].cpu().numpy(), S) <= TOL_BF16
    # state-only (first phase of the sequence-parallel scan): no q, no o
    _, S2, dec2, _ = m.ops.gated_scan_fwd(None, k.cuda(), v.cuda(), f.cuda(), want_final=True,
                                          want_output=False)
    # pass-1 (state-only) and pass-2 state paths round bf16 operands differently
    assert float((S2 - S_fin).abs().max() / S_fin.abs().max()) <= TOL_BF16
    assert torch.allclose(dec2, dec)


def test_repeated_calls_reuse_workspace(mg):
    m, N = mg
    q, k, v, f = (t.cuda() for t in headed_bf16(1, 4, 3000, seed=2))
    outs = [m.gated_scan(q, k, v, f) for _ in range(4)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert all(e == 0 for e in N.workspace_errors())


def test_full_length_split_consistency(mg):
    """Config 2 at full length: scanning [0, T) equals scanning [0, T/2) then
    [T/2, T) from the carried state (a size-independent property), and the
    first 2048 steps match the oracle."""
    m, _ = mg
    T = 32768
    q, k, v, f = (t.cuda() for t in headed_bf16(1, 12, T, seed=3))
    o = m.gated_scan(q, k, v, f, output_dtype=torch.float32)
    # split at a chunk boundary: identical chunking on both sides, so only the
    # carry path differs (fp32 sums in another order, bf16 state operands
    # rounded at other chunks); bounded well inside the 2e-2 bf16 tolerance
    h = T // 2 + 64 * 7
    o1, S1, _, _ = m.ops.gated_scan_fwd(q[:, :, :h], k[:, :, :h], v[:, :, :h], f[:, :, :h],
                                        output_dtype=torch.float32, want_final=True)
    o2, _, _, _ = m.ops.gated_scan_fwd(q[:, :, h:], k[:, :, h:], v[:, :, h:], f[:, :, h:],
                                       initial_state=S1, output_dtype=torch.float32)
    both = torch.cat([o1, o2], 2)
    err = (both - o).abs().max() / o.abs().max()
    assert float(err) <= 5e-3
    ref = O.gated_scan(*as64(q[:1, :2, :2048], k[:1, :2, :2048], v[:1, :2, :2048], f[:1, :2, :2048]))
    assert rel_max_err(o[:1, :2, :2048].cpu().numpy(), ref) <= TOL_BF16
    assert torch.isfinite(o).all()


def test_errors(mg):
    m, _ = mg
    q, k, v, f = headed_bf16(1, 1, 16)
    with pytest.raises(ValueError):
        m.gated_scan(q, k, v, f)  # CPU tensors: no fallback
    with pytest.raises(ValueError):
        m.gated_scan(q.cuda()[..., :32], k.cuda()[..., :32], v.cuda()[..., :32], f.cuda())
    with pytest.raises(ValueError):
        m.gated_scan(q.cuda(), k.cuda(), v.cuda(), f.cuda()[..., :8])


@pytest.mark.parametrize("H,T", [(12, 3584), (12, 5000), (12, 6000), (1, 5000)])
def test_every_output_row_written(mg, H, T):
    """Outputs prefilled with NaN: every row of every stripe must be written
    (stripes of 5 to 8 chunks at H = 12, one stripe per chunk at H = 1), and
    must match the oracle."""
    m, N = mg
    q, k, v, f = headed_bf16(1, H, T, seed=21)
    qc, kc, vc, fc = (t.cuda() for t in (q, k, v, f))
    L = N.lib()
    nb = L.mogt_gated_scan_fwd_workspace_bytes(H, T, 64, 64, N.BF16)
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    o = torch.full((1, H, T, 64), float("nan"), dtype=torch.float32, device="cuda")
    st = L.mogt_gated_scan_fwd(N.ptr(qc), N.ptr(kc), N.ptr(vc), N.ptr(fc), N.ptr(o), None, None, None, None,
                               H, T, 64, 64, N.BF16, N.F32, N.ptr(ws), nb, N.stream_ptr(qc.device))
    assert st == 0
    assert torch.isfinite(o).all()
    ref = O.gated_scan(*as64(q, k, v, f))
    assert rel_max_err(o.cpu().numpy(), ref) <= TOL_BF16


@pytest.mark.parametrize("T", [700, 9000])
def test_resume_after_state_only_pass(mg, T):
    """mogt_gated_scan_fwd_resume (the sequence-parallel scan's second pass):
    a state-only forward, then the output pass resumed from an initial state,
    equals one forward from that state, and its final state and decay equal
    the state-only pass's carried through that state."""
    from mogt_b200 import ops
    q, k, v, f = (t.cuda() for t in headed_bf16(2, 3, T, seed=11 + T))
    S0 = torch.randn(2, 3, 64, 64, generator=torch.Generator().manual_seed(T)).cuda()
    _, S_loc, A_loc, _ = ops.gated_scan_fwd(None, k, v, f, want_final=True, want_output=False)
    o_r, S_r, A_r, _ = ops.gated_scan_fwd(q, k, v, f, initial_state=S0, want_final=True, resume=True)
    o_f, S_f, A_f, _ = ops.gated_scan_fwd(q, k, v, f, initial_state=S0, want_final=True)
    assert rel_max_err(o_r.float().cpu().numpy(), o_f.float().cpu().numpy()) <= 1e-2
    assert torch.allclose(A_r, A_f) and torch.allclose(A_loc, A_f)
    carried = A_loc[..., None, None] * S0 + S_loc
    assert rel_max_err(S_r.cpu().numpy(), carried.cpu().numpy()) <= 1e-4
    assert rel_max_err(S_r.cpu().numpy(), S_f.cpu().numpy()) <= 1e-5
    ref = O.gated_scan(*as64(q, k, v, f), S0=as64(S0)[0])
    assert rel_max_err(o_r.float().cpu().numpy(), ref) <= TOL_BF16


def test_mixed_gates_across_multi_chunk_segments(mg):
    """Exact-decay chunks (zero, one and tiny gates) inside segments of several
    chunks (BH = 2, T = 65536: five chunks per segment of the local pass),
    with an initial state: outputs, final state and decay, and the saved
    state entering sampled chunks, against the float64 oracle."""
    m, _ = mg
    T = 65536
    q, k, v, f = headed_bf16(1, 2, T, seed=21, f_mode="mixed")
    S0 = torch.randn(1, 2, 64, 64, generator=torch.Generator().manual_seed(3))
    o, S_fin, dec, seg = m.ops.gated_scan_fwd(q.cuda(), k.cuda(), v.cuda(), f.cuda(),
                                              initial_state=S0.cuda(), output_dtype=torch.float32,
                                              want_final=True, save_states=True)
    q64, k64, v64, f64 = as64(q, k, v, f)
    ref, Sref = O.gated_scan(q64, k64, v64, f64, S0=S0.double().numpy(), return_final=True)
    assert rel_max_err(o.cpu().numpy(), ref) <= TOL_BF16
    assert rel_max_err(S_fin.cpu().numpy(), Sref) <= TOL_BF16
    assert np.allclose(dec.cpu().numpy(), np.prod(f64, axis=-1), rtol=1e-3, atol=1e-30)
    for c in (1, 5, 6, 333, 1023):
        _, Sc = O.gated_scan(q64[:, :, :64 * c], k64[:, :, :64 * c], v64[:, :, :64 * c],
                             f64[:, :, :64 * c], S0=S0.double().numpy(), return_final=True)
        assert rel_max_err(seg[:, :, c].float().cpu().numpy(), Sc) <= TOL_BF16


def test_resume_refused_without_matching_state_only_pass(mg):
    """A resumed output pass needs the chunk-local states of the same k, v, f
    in the workspace: after a call that kept its states elsewhere
    (save_states) or after a forward of other inputs it is refused."""
    from mogt_b200 import ops
    q, k, v, f = (t.cuda() for t in headed_bf16(1, 2, 700, seed=31))
    ops.gated_scan_fwd(q, k, v, f, save_states=True)
    with pytest.raises(ValueError, match="resume"):
        ops.gated_scan_fwd(q, k, v, f, resume=True)
    ops.gated_scan_fwd(None, k, v, f, want_final=True, want_output=False)
    k2 = k.clone()
    with pytest.raises(ValueError, match="resume"):
        ops.gated_scan_fwd(q, k2, v, f, resume=True)
    o, _, _, _ = ops.gated_scan_fwd(q, k, v, f, resume=True)
    assert torch.equal(o, ops.gated_scan_fwd(q, k, v, f)[0])
