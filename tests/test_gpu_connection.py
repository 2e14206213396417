"""Connection-map kernel (mogt_connection_map) against the reference's own
formula (model_mogt.py:79-102, 132-133: A = M - M^T in the input dtype, then
torch.matrix_exp or the Cayley solve of A / r in fp32), evaluated here in
float64 with torch; gradients against torch autograd in float64.
Tolerance: fp32 arithmetic, 1e-5 relative (max-abs error over max-abs)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _ref(M, impl, damping):
    r = M.shape[-1]
    A = (M - M.transpose(-1, -2)).double() / r
    if impl == "matrix_exp":
        U = torch.matrix_exp(A)
    else:
        eye = torch.eye(r, dtype=torch.float64, device=M.device)
        U = torch.linalg.solve(eye - 0.5 * A, eye + 0.5 * A)
    return U * damping


def _rel(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max())


@pytest.mark.parametrize("impl", ["matrix_exp", "cayley"])
@pytest.mark.parametrize("scale", [1e-4, 0.3, 8.0])
@pytest.mark.parametrize("r", [8, 16])
def test_forward_matches_reference_formula(impl, scale, r):
    from mogt_b200.connection import connection_map
    g = torch.Generator(device="cuda").manual_seed(int(scale * 1000) + r)
    M = scale * torch.randn(3, 257, r, r, generator=g, device="cuda")
    U = connection_map(M, impl, damping=0.999, output_dtype=torch.float32)
    assert _rel(U, _ref(M, impl, 0.999)) <= TOL


@pytest.mark.parametrize("impl", ["matrix_exp", "cayley"])
def test_bf16_input_rounds_like_the_reference(impl):
    from mogt_b200.connection import connection_map
    g = torch.Generator(device="cuda").manual_seed(3)
    M = (0.5 * torch.randn(2, 100, 16, 16, generator=g, device="cuda")).bfloat16()
    U = connection_map(M, impl, damping=0.999, output_dtype=torch.float32)
    # the reference forms A_raw - A_raw^T in bf16 (autocast), then maps in fp32
    assert _rel(U, _ref(M, impl, 0.999)) <= TOL
    Ub = connection_map(M, impl, damping=0.999)
    assert Ub.dtype == torch.bfloat16 and _rel(Ub, _ref(M, impl, 0.999)) <= 1e-2


@pytest.mark.parametrize("impl", ["matrix_exp", "cayley"])
def test_gradients_match_autograd(impl):
    from mogt_b200.connection import connection_map
    g = torch.Generator(device="cuda").manual_seed(5)
    M = 0.7 * torch.randn(4, 33, 16, 16, generator=g, device="cuda")
    G = torch.randn(4, 33, 16, 16, generator=g, device="cuda")
    Mc = M.clone().requires_grad_(True)
    (dM,) = torch.autograd.grad(connection_map(Mc, impl, damping=0.999), Mc, grad_outputs=G)
    Md = M.double().requires_grad_(True)
    (dMr,) = torch.autograd.grad(_ref(Md, impl, 0.999), Md, grad_outputs=G.double())
    assert _rel(dM, dMr) <= 1e-4


def test_backbone_matrix_exp_connection():
    """The backbone's default connection (matrix_exp) through the kernel:
    the same model with the oracle scan agrees (both use the kernel for U)."""
    from tests.test_gpu_backbone import _models
    a, b = _models()
    for m in (a, b):
        for blk in m.blocks:
            blk.connection_impl = "matrix_exp"
            torch.nn.init.normal_(blk.phi_conn.weight, std=0.05)
    b.load_state_dict(a.state_dict())
    ids = torch.randint(0, 300, (2, 500), device="cuda")
    with torch.inference_mode():
        ya, yb = a(ids), b(ids)
    assert float((ya - yb).abs().max() / yb.abs().max()) <= 1e-4
