"""Backward of the fused diagonal scan + RMSNorm (mogt_diag_scan_norm_bwd)
against torch autograd through the dense formulation the reference trains
with (U = damping (1 - z) I, V * z, the affine scan, norm_out), in float64.
fp32 arithmetic: 1e-4 relative for fp32 V, 2e-2 for bf16 V."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dense_ref(V, z, w, damping, eps, H0=None):
    """h_t = damping (1 - z_t) h_{t-1} + V_t z_t per row, y = RMSNorm(h) w (float64)."""
    B, L, R, C = V.shape
    h = torch.zeros(B, R, C, dtype=torch.float64, device=V.device) if H0 is None else H0
    ys = []
    for t in range(L):
        zt = z[:, t].view(B, -1, 1)
        h = damping * (1 - zt) * h + V[:, t] * zt
        hf = h.reshape(B, R * C)
        ys.append(hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps) * w)
    return torch.stack(ys, 1)


@pytest.mark.parametrize("L,zs,dtype", [(37, 16, torch.float32), (300, 16, torch.float32),
                                        (300, 1, torch.float32), (513, 16, torch.bfloat16)])
def test_gradients_match_dense_autograd(L, zs, dtype):
    from mogt_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(L + zs)
    B, R, C = 2, 16, 48
    V = torch.randn(B, L, R, C, generator=g, device="cuda").to(dtype)
    z = torch.sigmoid(torch.randn(B, L, zs, 1, generator=g, device="cuda") - 1.0)
    w = 1 + 0.1 * torch.randn(R * C, generator=g, device="cuda")
    H0 = torch.randn(B, R, C, generator=g, device="cuda")
    dy = torch.randn(B, L, R * C, generator=g, device="cuda")
    damping, eps = 0.999, 1e-6
    leaves = [V.clone().requires_grad_(True), z.clone().requires_grad_(True), w.clone().requires_grad_(True),
              H0.clone().requires_grad_(True)]
    y = ops.DiagScanNormFn.apply(leaves[0], leaves[1], leaves[2], leaves[3], damping, eps, torch.float32)
    got = torch.autograd.grad(y, leaves, grad_outputs=dy)
    refl = [t.detach().double().requires_grad_(True) for t in (V, z, w, H0)]
    yr = _dense_ref(refl[0], refl[1], refl[2], damping, eps, refl[3])
    assert float((y.detach().double() - yr.detach()).abs().max() / yr.abs().max()) <= (1e-4 if dtype == torch.float32 else 2e-2)
    ref = torch.autograd.grad(yr, refl, grad_outputs=dy.double())
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    for name, a, b in zip(("dV", "dz", "dw", "dH0"), got, ref):
        err = float((a.double() - b).abs().max() / b.abs().max())
        assert err <= tol, (name, err)


def test_backbone_training_step_uses_fused_backward():
    """A training step of the identity-coupled backbone through the fused
    forward/backward matches the same model on the dense path."""
    from mogt_b200.backbone import MOGTModel, configure_identity_coupled
    torch.manual_seed(0)
    a = MOGTModel(300, 128, 2, 16)
    for p in a.parameters():
        torch.nn.init.normal_(p, std=0.02)
    configure_identity_coupled(a)
    for blk in a.blocks:
        torch.nn.init.normal_(blk.phi_value_gate.weight, std=0.02)
    b = MOGTModel(300, 128, 2, 16)
    configure_identity_coupled(b)
    b.load_state_dict(a.state_dict())
    for blk in b.blocks:
        blk.fused_identity_scan = False  # dense U + affine scan autograd
    a, b = a.cuda(), b.cuda()
    ids = torch.randint(0, 300, (2, 400), device="cuda")
    grads = []
    for m in (a, b):
        out = m(ids)
        loss = out.float().pow(2).mean()
        grads.append(torch.autograd.grad(loss, [m.blocks[0].phi_val.weight, m.blocks[0].phi_value_gate.weight,
                                                m.blocks[1].norm_out.weight]))
    for ga, gb in zip(*grads):
        assert float((ga - gb).abs().max() / gb.abs().max()) <= 1e-3
