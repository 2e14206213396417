"""MOGT backbone with the CUDA scan vs the same model with the oracle's
sequential scan (fp32), and under bf16 autocast (the benchmark's setting)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _oracle_scan(U, V, out_dtype):
    from oracle import scan_oracle as O
    H = O.affine_scan_sequential(U.detach().double().cpu().numpy(), V.detach().double().cpu().numpy())
    return torch.from_numpy(H).to(device=U.device, dtype=out_dtype)


def _models(d=128, r=16, layers=2, vocab=300):
    from mogt_b200.backbone import MOGTModel, configure_identity_coupled
    torch.manual_seed(0)
    a = MOGTModel(vocab, d, layers, r)
    for p in a.parameters():
        torch.nn.init.normal_(p, std=0.02)
    configure_identity_coupled(a)
    for blk in a.blocks:
        torch.nn.init.normal_(blk.phi_value_gate.weight, std=0.02)
    b = MOGTModel(vocab, d, layers, r, scan_fn=_oracle_scan)
    configure_identity_coupled(b)
    b.load_state_dict(a.state_dict())
    return a.cuda().eval(), b.cuda().eval()


@pytest.mark.parametrize("connection", ["identity", "cayley"])
def test_backbone_cuda_scan_matches_oracle_scan(connection):
    a, b = _models()
    for m in (a, b):
        for blk in m.blocks:
            blk.connection_impl = connection
    ids = torch.randint(0, 300, (2, 700), device="cuda")
    with torch.inference_mode():
        ya, yb = a(ids), b(ids)
    err = float((ya - yb).abs().max() / yb.abs().max())
    assert err <= 1e-4


def test_backbone_bf16_autocast():
    a, b = _models()
    ids = torch.randint(0, 300, (1, 1000), device="cuda")
    with torch.inference_mode():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            ya = a(ids)
        yb = b(ids)
    assert torch.isfinite(ya.float()).all()
    err = float((ya.float() - yb).abs().max() / yb.abs().max())
    assert err <= 2e-2
