"""Pin the numpy oracle against the reference's own outputs (golden vectors
made by tests/golden/make_golden.py from affine_scan.py) and against the
reference sanity script's identities (sanity_affine_scan.py:19-61, 102-135)."""
import numpy as np
import pytest

from oracle import scan_oracle as O
from tests.golden.make_golden import headed_inputs


def test_sanity_identities_match_reference(golden):
    d = golden("sanity_r4")
    U, V = d["U"], d["V"]
    kw = dict(state_dtype=np.float64, output_dtype=np.float64, return_prefix=True)
    Ps, Hs = O.affine_scan_sequential(U, V, **kw)
    Pd, Hd = O.affine_scan_doubling(U, V, **kw)
    Pb, Hb = O.affine_scan_block_reference(U, V, block_size=5, carry_scan="doubling", **kw)
    tol = 1e-10  # sanity_affine_scan.py:57
    for mine, ref in [(Ps, d["P_seq"]), (Hs, d["H_seq"]), (Pd, d["P_dbl"]), (Hd, d["H_dbl"]),
                      (Pb, d["P_blk"]), (Hb, d["H_blk"])]:
        assert np.abs(mine - ref).max() < tol
    assert np.abs(Ps - Pd).max() < tol and np.abs(Hs - Hb).max() < tol


def test_sequential_backward_matches_reference(golden):
    d = golden("sanity_r4")
    gU, gV = O.affine_scan_sequential_backward(d["U_bwd"], d["V_bwd"], d["g_bwd"])
    assert np.abs(gU - d["gU"]).max() < 1e-10
    assert np.abs(gV - d["gV"]).max() < 1e-10


@pytest.mark.parametrize("name", ["native_r16_c8_l64", "native_r16_c48_l70"])
def test_native_shape_fp32_matches_reference(golden, name):
    d = golden(name)
    P, H = O.affine_scan_sequential(d["U"], d["V"], state_dtype=np.float32,
                                    output_dtype=np.float32, return_prefix=True)
    # same fp32 arithmetic, different BLAS: agreement to fp32 round-off
    assert np.abs(H - d["H"]).max() <= 1e-5 * max(1.0, np.abs(d["H"]).max())
    assert np.abs(P - d["P"]).max() <= 1e-5
    gU, gV = O.affine_scan_sequential_backward(d["U"], d["V"], d["g"], state_dtype=np.float32)
    assert np.abs(gV - d["gV"]).max() <= 1e-5 * np.abs(d["gV"]).max()
    assert np.abs(gU - d["gU"]).max() <= 1e-5 * np.abs(d["gU"]).max()


def test_block_with_ragged_last_block():
    rng = np.random.default_rng(3)
    U = np.eye(4) + 0.05 * rng.standard_normal((2, 23, 4, 4))
    V = rng.standard_normal((2, 23, 4, 5))
    H = O.affine_scan_sequential(U, V)
    for bs in (1, 4, 7, 23, 64):
        for cs in ("sequential", "doubling"):
            assert np.abs(O.affine_scan_block_reference(U, V, block_size=bs, carry_scan=cs) - H).max() < 1e-12


def test_headed_small_fp64_matches_reference(golden):
    d = golden("headed_small_fp64")
    o = O.gated_scan(d["q"], d["k"], d["v"], d["f"])
    od = O.gated_scan_dense(d["q"], d["k"], d["v"], d["f"])
    assert np.abs(o - d["o"]).max() < 1e-12
    assert np.abs(od - d["o"]).max() < 1e-12
    dq, dk, dv, df = O.gated_scan_backward(d["q"], d["k"], d["v"], d["f"], d["g"])
    for mine, key in [(dq, "dq"), (dk, "dk"), (dv, "dv"), (df, "df")]:
        assert np.abs(mine - d[key]).max() < 1e-10, key


def test_scalar_gate_equals_dense_gate_fp32():
    """f*S and (f I) @ S give the same fp32 numbers: the scalar-gate oracle is
    the dense reference operator, not an approximation of it."""
    q, k, v, f, _ = (x.numpy() for x in headed_inputs(1, 2, 33, 8, 8, __import__("torch").float32))
    a = O.gated_scan(q, k, v, f, state_dtype=np.float32)
    b = O.gated_scan_dense(q, k, v, f, state_dtype=np.float32)
    assert np.abs(a - b).max() <= 1e-6 * np.abs(b).max()


def test_config1_matches_reference(golden):
    import torch
    d = golden("config1_fp32")
    q, k, v, f, g = headed_inputs(2, 4, 512, 32, 32, torch.float32)
    assert abs(sum(float(x.double().sum()) for x in (q, k, v, f, g)) - float(d["input_checksum"])) < 1e-9
    q, k, v, f, g = (x.numpy() for x in (q, k, v, f, g))
    o = O.gated_scan(q, k, v, f, state_dtype=np.float32)
    scale = np.abs(d["o"]).max()
    assert np.abs(o - d["o"]).max() <= 1e-5 * scale
    o64 = O.gated_scan(q, k, v, f)
    assert np.abs(o64 - d["o"]).max() <= 1e-5 * scale
    dq, dk, dv, df = O.gated_scan_backward(q, k, v, f, g)
    for mine, key in [(dq, "dq"), (dk, "dk"), (dv, "dv"), (df, "df")]:
        ref = d[key]
        assert np.abs(mine - ref).max() <= 1e-4 * np.abs(ref).max(), key


def test_matrix_small_fp64_matches_reference(golden):
    d = golden("matrix_small_fp64")
    o = O.matrix_scan(d["A"], d["q"], d["k"], d["v"], d["f"])
    assert np.abs(o - d["o"]).max() < 1e-12
    dA, dq, dk, dv, df = O.matrix_scan_backward(d["A"], d["q"], d["k"], d["v"], d["f"], d["g"])
    for mine, key in [(dA, "dA"), (dq, "dq"), (dk, "dk"), (dv, "dv"), (df, "df")]:
        assert np.abs(mine - d[key]).max() < 1e-10, key


def test_initial_state_and_final_state():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 2, 30, 4)) for _ in range(3))
    f = 1 / (1 + np.exp(-rng.standard_normal((1, 2, 30)) - 2))
    o_full, S_full = O.gated_scan(q, k, v, f, return_final=True)
    o1, S1 = O.gated_scan(q[:, :, :11], k[:, :, :11], v[:, :, :11], f[:, :, :11], return_final=True)
    o2, S2 = O.gated_scan(q[:, :, 11:], k[:, :, 11:], v[:, :, 11:], f[:, :, 11:], S0=S1, return_final=True)
    assert np.abs(np.concatenate([o1, o2], 2) - o_full).max() < 1e-12
    assert np.abs(S2 - S_full).max() < 1e-12
    od = O.gated_scan_dense(q[:, :, 11:], k[:, :, 11:], v[:, :, 11:], f[:, :, 11:], S0=S1)
    assert np.abs(od - o2).max() < 1e-12


def test_oracle_shape_errors():
    with pytest.raises(ValueError):
        O.affine_scan_sequential(np.zeros((1, 2, 3, 3)), np.zeros((1, 2, 4, 3)))
    with pytest.raises(ValueError):
        O.affine_scan_sequential(np.zeros((2, 3, 3)), np.zeros((1, 2, 3, 3)))


def test_streaming_matrix_forms_match_dense_oracle(golden):
    """The streaming dense-transition forms used by the full-size checks equal
    the dense composition (itself pinned to the reference's vectors)."""
    d = golden("matrix_small_fp64")
    A, q, k, v, f = (d[x] for x in ("A", "q", "k", "v", "f"))
    o = O.matrix_scan_stream(A, q, k, v, f)
    assert np.abs(o - d["o"]).max() <= 1e-10 * max(1.0, np.abs(d["o"]).max())
    stream = O.matrix_scan_backward_stream(A, q, k, v, f, d["g"], chunk=7)
    for name, b in zip(("dA", "dq", "dk", "dv", "df"), stream[:5]):
        a = d[name]
        assert np.abs(a - b).max() <= 1e-6 * np.abs(a).max(), name


def test_torch_reference_path_matches_oracle():
    """The torch form timed as the CPU baseline computes the oracle's result."""
    from tests.helpers import as64, headed_bf16
    q, k, v, f = headed_bf16(1, 3, 130, seed=4)
    o = O.gated_scan_torch_reference_path(q.float(), k.float(), v.float(), f)
    r = O.gated_scan(*as64(q, k, v, f))
    assert np.abs(o.numpy() - r).max() <= 1e-5 * np.abs(r).max()


def test_chunked_ce_golden_is_plain_cross_entropy(golden):
    """The reference-made chunked CE golden equals torch's cross-entropy over
    the whole batch (loss and ignored-label handling), on the CPU."""
    import torch
    d = golden("chunked_ce")
    h = torch.from_numpy(d["hidden"]).double()
    w = torch.from_numpy(d["weight"]).double()
    lab = torch.from_numpy(d["labels"]).reshape(-1)
    logits = h.reshape(-1, h.shape[-1]) @ w.t()
    ref = torch.nn.functional.cross_entropy(logits, lab, reduction="sum") / lab.numel()
    assert abs(float(ref) - float(d["loss"])) <= 1e-5 * abs(float(ref))
