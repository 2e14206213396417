"""Dense affine scan (the reference operator's native form) on the GPU:
mogt_b200.triton_scan against golden vectors from the reference and the
oracle.  fp32 state, fp32 tolerance 1e-4 relative (the reference's own
Triton check uses 5e-5 absolute at L=64, sanity_affine_scan.py:64-99)."""
import numpy as np
import pytest
import torch

from oracle import scan_oracle as O
from tests.helpers import rel_max_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(scope="module")
def ts():
    from mogt_b200 import triton_scan
    return triton_scan


def _uv(B, L, R, C, seed=0, scale=0.05, vdtype=torch.float32, diag=1.0):
    """U = diag * I + scale * N(0,1); diag < 1 keeps long products bounded."""
    g = torch.Generator().manual_seed(seed)
    U = diag * torch.eye(R) + scale * torch.randn(B, L, R, R, generator=g)
    V = torch.randn(B, L, R, C, generator=g).to(vdtype)
    return U, V


@pytest.mark.parametrize("name", ["native_r16_c8_l64", "native_r16_c48_l70"])
def test_golden_forward_and_backward(ts, golden, name):
    d = golden(name)
    U, V, g = (torch.from_numpy(d[x]).cuda() for x in ("U", "V", "g"))
    P, H = ts.triton_affine_scan_hybrid(U, V, output_dtype=torch.float32, return_prefix=True)
    assert rel_max_err(H.cpu().numpy(), d["H"]) <= TOL
    assert rel_max_err(P.cpu().numpy(), d["P"]) <= TOL
    Ur, Vr = U.clone().requires_grad_(True), V.clone().requires_grad_(True)
    Ho = ts.triton_affine_scan_hybrid(Ur, Vr, block_size=32, block_c=8, output_dtype=torch.float32)
    gU, gV = torch.autograd.grad(Ho, (Ur, Vr), grad_outputs=g)
    assert rel_max_err(gV.cpu().numpy(), d["gV"]) <= TOL
    assert rel_max_err(gU.cpu().numpy(), d["gU"]) <= TOL


def test_sanity_r4_golden(ts, golden):
    d = golden("sanity_r4")
    U = torch.from_numpy(d["U"]).float().cuda()
    V = torch.from_numpy(d["V"]).float().cuda()
    # C = 3 columns, R = 4
    P, H = ts.triton_affine_scan_hybrid(U, V, output_dtype=torch.float32, return_prefix=True)
    assert rel_max_err(H.cpu().numpy(), d["H_seq"]) <= 1e-5
    assert rel_max_err(P.cpu().numpy(), d["P_seq"]) <= 1e-5


@pytest.mark.parametrize("B,L,R,C", [(1, 1, 16, 48), (2, 31, 16, 48), (1, 33, 16, 48), (3, 1000, 16, 48),
                                     (1, 5000, 16, 8), (2, 300, 8, 24), (1, 700, 4, 3), (1, 400, 32, 16),
                                     (1, 129, 2, 5)])
def test_forward_vs_oracle(ts, B, L, R, C):
    U, V = _uv(B, L, R, C, seed=L + R, scale=0.1 / R ** 0.5, diag=0.95)
    P, H = ts.triton_affine_scan_hybrid(U.cuda(), V.cuda(), output_dtype=torch.float32, return_prefix=True)
    Pr, Hr = O.affine_scan_sequential(U.double().numpy(), V.double().numpy(), return_prefix=True)
    assert rel_max_err(H.cpu().numpy(), Hr) <= TOL
    assert rel_max_err(P.cpu().numpy(), Pr) <= TOL


def test_model_dtypes_fp32_U_bf16_V(ts):
    """Autocast path of MOGTBlock: U fp32, V bf16, output fp32 (model_mogt.py:196-203)."""
    U, V = _uv(2, 2000, 16, 48, seed=9, scale=0.02, vdtype=torch.bfloat16)
    H = ts.triton_affine_scan_hybrid(U.cuda(), V.cuda(), output_dtype=U.dtype)
    assert H.dtype == torch.float32
    Hr = O.affine_scan_sequential(U.double().numpy(), V.double().numpy())
    assert rel_max_err(H.cpu().numpy(), Hr) <= TOL
    Hb = ts.triton_affine_scan_hybrid(U.cuda(), V.cuda())  # default: V.dtype
    assert Hb.dtype == torch.bfloat16
    assert rel_max_err(Hb.float().cpu().numpy(), Hr) <= 1e-2


def test_diagonal_rank_gate_long(ts):
    """Backbone config: U = diag(1 - z) (identity connection, rank-wise coupled
    gate), L = 32768."""
    g = torch.Generator().manual_seed(4)
    z = torch.sigmoid(torch.randn(1, 32768, 16, generator=g) - 2.0)
    U = torch.diag_embed(1.0 - z)
    V = (torch.randn(1, 32768, 16, 48, generator=g) * z[..., None]).bfloat16()
    H = ts.triton_affine_scan_hybrid(U.cuda(), V.cuda(), output_dtype=torch.float32)
    Hr = O.affine_scan_sequential(U[:, :3000].double().numpy(), V[:, :3000].double().numpy())
    assert rel_max_err(H[:, :3000].cpu().numpy(), Hr) <= TOL
    # tail: independent recurrence from the kernel's own state at 30000
    s = 30000
    Ht = O.affine_scan_sequential(
        np.concatenate([np.zeros((1, 1, 16, 16)), U[:, s + 1:].double().numpy()], 1),
        np.concatenate([H[:, s:s + 1].double().cpu().numpy(), V[:, s + 1:].double().numpy()], 1))
    assert rel_max_err(H[:, s:].cpu().numpy(), Ht) <= TOL


def test_backward_vs_oracle(ts):
    U, V = _uv(2, 777, 16, 48, seed=1, scale=0.05)
    gH = torch.randn(2, 777, 16, 48)
    gU, gV = ts._triton_affine_scan_hybrid_backward(U.cuda(), V.cuda(), gH.cuda(), block_size=256,
                                                    block_c=32, carry_scan="sequential",
                                                    need_grad_u=True, need_grad_v=True)
    gUr, gVr = O.affine_scan_sequential_backward(U.double().numpy(), V.double().numpy(), gH.double().numpy())
    assert rel_max_err(gV.cpu().numpy(), gVr) <= TOL
    assert rel_max_err(gU.cpu().numpy(), gUr) <= TOL


def test_local_scan_and_fused_scan(ts):
    U, V = _uv(2, 100, 16, 8, seed=7)
    Up, Hp, Us, Hs = ts.triton_affine_local_scan(U.cuda(), V.cuda(), block_size=32, block_c=8)
    Pr, Hr = O.affine_scan_block_reference(U.double().numpy(), V.double().numpy(), block_size=32,
                                           return_prefix=True)
    # block-local prefixes: restart every 32 steps
    for b0 in range(0, 100, 32):
        b1 = min(b0 + 32, 100)
        Pl, Hl = O.affine_scan_sequential(U[:, b0:b1].double().numpy(), V[:, b0:b1].double().numpy(),
                                          return_prefix=True)
        assert rel_max_err(Hp[:, b0:b1].cpu().numpy(), Hl) <= TOL
        assert rel_max_err(Up[:, b0:b1].cpu().numpy(), Pl) <= TOL
        assert rel_max_err(Hs[:, b0 // 32].cpu().numpy(), Hl[:, -1]) <= TOL
        assert rel_max_err(Us[:, b0 // 32].cpu().numpy(), Pl[:, -1]) <= TOL
    Y = ts.triton_fused_scan(U.cuda())
    assert rel_max_err(Y.cpu().numpy(), Pr) <= TOL


def test_errors(ts):
    U, V = _uv(1, 8, 16, 4)
    with pytest.raises(ValueError):
        ts.triton_affine_local_scan(U, V)
    with pytest.raises(ValueError):
        ts.triton_affine_scan_hybrid(U.cuda()[..., :3], V.cuda())
    with pytest.raises(ValueError):
        ts.triton_affine_scan_hybrid(U.cuda(), V.cuda(), carry_scan="bogus")
