"""Dense-transition headed scan (config 3) against the golden vectors of the
reference and the oracle (tolerances: fp32 1e-4, bf16 inputs 2e-2)."""
import numpy as np
import pytest
import torch

from oracle import scan_oracle as O
from tests.helpers import as64, rel_max_err

pytestmark = pytest.mark.gpu


def _cayley(B, H, T, d, seed):
    g = torch.Generator().manual_seed(seed)
    M = torch.randn(B, H, T, d, d, generator=g, dtype=torch.float64)
    W = 0.05 * (M - M.transpose(-1, -2))
    I = torch.eye(d, dtype=torch.float64)
    return torch.linalg.solve(I - W, I + W).float()


def test_golden_small(golden):
    import mogt_b200
    d = golden("matrix_small_fp64")
    A, q, k, v, f = (torch.from_numpy(d[x]).float().cuda() for x in ("A", "q", "k", "v", "f"))
    o = mogt_b200.matrix_scan(A, q, k, v, f)
    assert rel_max_err(o.cpu().numpy(), d["o"]) <= 1e-4


@pytest.mark.parametrize("d,T", [(64, 300), (32, 129), (16, 1)])
def test_bf16_vs_oracle(d, T):
    import mogt_b200
    g = torch.Generator().manual_seed(d + T)
    q, k, v = (torch.randn(2, 2, T, d, generator=g).bfloat16() for _ in range(3))
    f = torch.sigmoid(torch.randn(2, 2, T, generator=g) + 2.0)
    A = _cayley(2, 2, T, d, seed=T)
    S0 = torch.randn(2, 2, d, d, generator=g)
    o, S = mogt_b200.ops.matrix_scan_fwd(A.cuda(), q.cuda(), k.cuda(), v.cuda(), f.cuda(),
                                         initial_state=S0.cuda(), output_dtype=torch.float32,
                                         want_final=True)
    # oracle with the initial state injected as a first step (U = 0, V = S0)
    Ad, qd, kd, vd, fd = as64(A, q, k, v, f)
    Bh = 4
    U = np.concatenate([np.zeros((Bh, 1, d, d)), Ad.reshape(Bh, T, d, d)], 1)
    Vin = (1 - fd.reshape(Bh, T))[..., None, None] * kd.reshape(Bh, T, d, 1) * vd.reshape(Bh, T, 1, d)
    Vin = np.concatenate([S0.double().numpy().reshape(Bh, 1, d, d), Vin], 1)
    Sref = O.affine_scan_sequential(U, Vin)[:, 1:]
    oref = np.einsum("ntkv,ntk->ntv", Sref, qd.reshape(Bh, T, d)).reshape(2, 2, T, d)
    assert rel_max_err(o.cpu().numpy(), oref) <= 1e-4
    assert rel_max_err(S.cpu().numpy(), Sref[:, -1].reshape(2, 2, d, d)) <= 1e-4


def test_config3_full_length_split_consistency():
    """Config 3 (B=2, H=8, T=8192, d=64): the full scan equals two halves
    joined through the carried state, and the first steps match the oracle."""
    import mogt_b200
    B, H, T, d = 2, 8, 8192, 64
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(B, H, T, d, generator=g).bfloat16().cuda() for _ in range(3))
    f = torch.sigmoid(torch.randn(B, H, T, generator=g) + 2.0).cuda()
    A = _cayley(B, H, T, d, seed=5).cuda()
    o, _ = mogt_b200.ops.matrix_scan_fwd(A, q, k, v, f, output_dtype=torch.float32)
    h = 4000
    o1, S1 = mogt_b200.ops.matrix_scan_fwd(A[:, :, :h], q[:, :, :h], k[:, :, :h], v[:, :, :h], f[:, :, :h],
                                           output_dtype=torch.float32, want_final=True)
    o2, _ = mogt_b200.ops.matrix_scan_fwd(A[:, :, h:], q[:, :, h:], k[:, :, h:], v[:, :, h:], f[:, :, h:],
                                          initial_state=S1, output_dtype=torch.float32)
    # the halves chunk at other boundaries (4000 is not a multiple of 64), so
    # the sums are formed in another order: the fp32 bar, not bit equality
    assert float((torch.cat([o1, o2], 2) - o).abs().max() / o.abs().max()) <= 1e-4
    oref = O.matrix_scan(*as64(A[:1, :2, :256], q[:1, :2, :256], k[:1, :2, :256], v[:1, :2, :256],
                               f[:1, :2, :256]))
    assert rel_max_err(o[:1, :2, :256].cpu().numpy(), oref) <= 1e-4


@pytest.mark.parametrize("T,dtype,precision", [(1, torch.bfloat16, "fp32"), (37, torch.bfloat16, "fp32"),
                                               (640, torch.bfloat16, "fp32"), (640, torch.float32, "fp32"),
                                               (1, torch.bfloat16, "tf32x3"), (37, torch.bfloat16, "tf32x3"),
                                               (64, torch.bfloat16, "tf32x3"), (640, torch.bfloat16, "tf32x3"),
                                               (1000, torch.bfloat16, "tf32x3")])
def test_chunked_vs_oracle_and_sequential(T, dtype, precision):
    """The chunked kernels (per-chunk prefix products and local states on the
    tensor cores for bf16 q/k/v, fp32 FMAs for fp32; chunk carries, per-chunk
    outputs; ragged last chunk) against the oracle and the single sequential
    pass.  The tensor-core form ("tf32x3") meets the fp32 bar up to ~1000
    steps; its accumulation bias grows with T (see the full-length test)."""
    d = 64
    import mogt_b200
    g = torch.Generator().manual_seed(7 * d + T)
    q, k, v = (torch.randn(1, 3, T, d, generator=g).to(dtype) for _ in range(3))
    f = torch.sigmoid(torch.randn(1, 3, T, generator=g) + 2.0)
    f[..., ::37] = 0.0
    A = _cayley(1, 3, T, d, seed=T + 1)
    S0 = torch.randn(1, 3, d, d, generator=g)
    args = (A.cuda(), q.cuda(), k.cuda(), v.cuda(), f.cuda())
    o, S = mogt_b200.ops.matrix_scan_fwd(*args, initial_state=S0.cuda(), output_dtype=torch.float32,
                                         want_final=True, chunked=True, precision=precision)
    o1, S1 = mogt_b200.ops.matrix_scan_fwd(*args, initial_state=S0.cuda(), output_dtype=torch.float32,
                                           want_final=True, chunked=False)
    assert rel_max_err(o.cpu().numpy(), o1.cpu().numpy()) <= 1e-4
    assert rel_max_err(S.cpu().numpy(), S1.cpu().numpy()) <= 1e-4
    Ad, qd, kd, vd, fd = as64(A, q, k, v, f)
    U = np.concatenate([np.zeros((3, 1, d, d)), Ad.reshape(3, T, d, d)], 1)
    Vin = (1 - fd.reshape(3, T))[..., None, None] * kd.reshape(3, T, d, 1) * vd.reshape(3, T, 1, d)
    Vin = np.concatenate([S0.double().numpy().reshape(3, 1, d, d), Vin], 1)
    Sref = O.affine_scan_sequential(U, Vin)[:, 1:]
    oref = np.einsum("ntkv,ntk->ntv", Sref, qd.reshape(3, T, d)).reshape(1, 3, T, d)
    assert rel_max_err(o.cpu().numpy(), oref) <= 1e-4
