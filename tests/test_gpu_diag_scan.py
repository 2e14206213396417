"""Fused diagonal gated scan + RMSNorm readout (the identity-connection MOGT
block) against the oracle: U = damping (1 - z) I and V * z.to(V.dtype) run
through the oracle's sequential affine scan in float64, then RMSNorm."""
import numpy as np
import pytest
import torch

from oracle import scan_oracle as O
from tests.helpers import rel_max_err

pytestmark = pytest.mark.gpu


def _inputs(B, L, R, C, dtype, row_gate, seed):
    g = torch.Generator().manual_seed(seed)
    V = torch.randn(B, L, R, C, generator=g).to(dtype)
    z = torch.sigmoid(torch.randn(B, L, R if row_gate else 1, 1, generator=g) - 1.0)
    w = 1.0 + 0.1 * torch.randn(R * C, generator=g)
    return V, z, w


def _reference(V, z, w, damping, eps, H0=None):
    """The reference block's arithmetic, in float64 from the rounded inputs."""
    B, L, R, C = V.shape
    zr = z.expand(B, L, R, 1)
    Vg = (V * zr.to(V.dtype)).double().numpy()                       # V * z.to(V.dtype)
    a = (np.float32(damping) * (1.0 - zr.float())).double().numpy()[..., 0]
    U = a[..., :, None] * np.eye(R)[None, None]
    if H0 is not None:
        U = np.concatenate([np.zeros((B, 1, R, R)), U], 1)
        Vg = np.concatenate([H0.double().numpy()[:, None], Vg], 1)
    H = O.affine_scan_sequential(U, Vg)
    if H0 is not None:
        H = H[:, 1:]
    Hf = H.reshape(B, L, R * C)
    y = Hf / np.sqrt((Hf ** 2).mean(-1, keepdims=True) + eps) * w.double().numpy()
    return y, H[:, -1]


@pytest.mark.parametrize("L", [1, 37, 64, 200, 1000])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_matches_oracle(L, dtype):
    from mogt_b200 import ops
    B, R, C = 2, 16, 48
    V, z, w = _inputs(B, L, R, C, dtype, True, seed=L)
    out_dtype = torch.bfloat16 if dtype == torch.bfloat16 else torch.float32
    y, Hf = ops.diag_scan_norm(V.cuda(), z.cuda(), w.cuda(), damping=0.999, eps=1e-6,
                               output_dtype=out_dtype, want_final=True)
    yr, Hr = _reference(V, z, w, 0.999, 1e-6)
    tol = 2e-2 if out_dtype == torch.bfloat16 else 1e-4
    assert y.dtype == out_dtype
    assert rel_max_err(y.float().cpu().numpy(), yr) <= tol
    assert rel_max_err(Hf.cpu().numpy(), Hr) <= 1e-4


def test_scalar_gate_initial_state_and_small_width():
    """One gate per token, an initial state, D = 128 (R = 16, C = 8)."""
    from mogt_b200 import ops
    B, L, R, C = 3, 300, 16, 8
    V, z, w = _inputs(B, L, R, C, torch.float32, False, seed=4)
    H0 = torch.randn(B, R, C, generator=torch.Generator().manual_seed(5))
    y, Hf = ops.diag_scan_norm(V.cuda(), z.cuda(), w.cuda(), damping=1.0, initial_state=H0.cuda(),
                               want_final=True)
    yr, Hr = _reference(V, z, w, 1.0, 1e-6, H0)
    assert rel_max_err(y.cpu().numpy(), yr) <= 1e-4
    assert rel_max_err(Hf.cpu().numpy(), Hr) <= 1e-4


def test_long_sequence_split_consistency():
    """L = 32768 (the backbone length): the scan equals two halves joined
    through the carried state (size-independent check of the chunk carries)."""
    from mogt_b200 import ops
    B, L, R, C = 2, 32768, 16, 48
    V, z, w = (t.cuda() for t in _inputs(B, L, R, C, torch.bfloat16, True, seed=9))
    y, Hf = ops.diag_scan_norm(V, z, w, output_dtype=torch.float32, want_final=True)
    h = 12345
    y1, H1 = ops.diag_scan_norm(V[:, :h], z[:, :h], w, output_dtype=torch.float32, want_final=True)
    y2, H2 = ops.diag_scan_norm(V[:, h:], z[:, h:], w, output_dtype=torch.float32, initial_state=H1,
                                want_final=True)
    assert float((torch.cat([y1, y2], 1) - y).abs().max() / y.abs().max()) <= 1e-4
    assert float((H2 - Hf).abs().max() / Hf.abs().max()) <= 1e-4
    yr, _ = _reference(V[:1, :300].cpu(), z[:1, :300].cpu(), w.cpu(), 1.0, 1e-6)
    assert rel_max_err(y[:1, :300].cpu().numpy(), yr) <= 1e-4


def test_block_fused_path_matches_unfused():
    """MOGTBlock under inference + bf16 autocast: the fused kernel path and
    the dense-U path through triton_affine_scan_hybrid agree."""
    from mogt_b200.backbone import MOGTModel, configure_identity_coupled
    torch.manual_seed(0)
    m = MOGTModel(500, 768, 2, 16)
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.02)
    configure_identity_coupled(m)
    for blk in m.blocks:
        torch.nn.init.normal_(blk.phi_value_gate.weight, std=0.05)
    m = m.cuda().eval()
    ids = torch.randint(0, 500, (2, 3000), device="cuda")
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        y_fused = m(ids).float()
        for blk in m.blocks:
            blk.fused_identity_scan = False
        y_dense = m(ids).float()
    err = float((y_fused - y_dense).abs().max() / y_dense.abs().max())
    assert err <= 2e-2, err


@pytest.mark.parametrize("mode", ["current", "current_prev", "current_prev_prefix"])
def test_gate_logits_match_concatenated_linear(mode):
    """The block's gate logits without the [x_t, x_{t-1}, x_prefix]
    concatenation equal phi_value_gate on the concatenation, under bf16
    autocast (one bf16 rounding apart at most) and in fp32."""
    from mogt_b200.backbone import MOGTBlock
    torch.manual_seed(3)
    blk = MOGTBlock(256, 16).cuda()
    mult = {"current": 1, "current_prev": 2, "current_prev_prefix": 3}[mode]
    blk.phi_value_gate = torch.nn.Linear(mult * 256, 16).cuda()
    blk.value_gate_input_mode = mode
    x = torch.randn(2, 500, 256, device="cuda")
    prefix = torch.randn(2, 256, device="cuda")
    with torch.inference_mode():
        for ac in (True, False):
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=ac):
                ref = blk.phi_value_gate(blk.value_gate_input(x, prefix)).float()
                got = blk._gate_logits(x, prefix, blk.phi_value_gate)
            tol = 1e-2 if ac else 1e-5
            assert float((got - ref).abs().max()) <= tol * float(ref.abs().max()), (mode, ac)


def test_wide_fp32_short_chunks():
    """D = 2048 fp32: the V tile budget cuts chunks to 8 tokens (pieces of 2
    tokens, shorter than a normalisation group); ragged L."""
    from mogt_b200 import ops
    B, L, R, C = 2, 101, 32, 64
    V, z, w = _inputs(B, L, R, C, torch.float32, True, seed=12)
    y, Hf = ops.diag_scan_norm(V.cuda(), z.cuda(), w.cuda(), damping=0.99, want_final=True)
    yr, Hr = _reference(V, z, w, 0.99, 1e-6)
    assert rel_max_err(y.cpu().numpy(), yr) <= 1e-4
    assert rel_max_err(Hf.cpu().numpy(), Hr) <= 1e-4
