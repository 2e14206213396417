"""The re-implemented MOGT backbone against the reference MOGTModel itself
(model_mogt.py), CPU only: the reference tree (MOGT_REFERENCE_DIR) is imported
read-only and the test is skipped where it is absent.  Weights are
copied from the reference model (same parameter names), the scan on both
sides is the reference's sequential affine scan (affine_scan.py:14-62), so
this pins the block and model plumbing around the scan."""
import os
import sys
from pathlib import Path

import pytest
import torch

REF = Path(os.environ["MOGT_REFERENCE_DIR"]) if os.environ.get("MOGT_REFERENCE_DIR") else None
pytestmark = pytest.mark.skipif(REF is None or not (REF / "model_mogt.py").exists(),
                                reason="reference tree absent (set MOGT_REFERENCE_DIR)")


def _ref_modules():
    sys.dont_write_bytecode = True
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import affine_scan
    import model_mogt
    return affine_scan, model_mogt


def _configure_ref(model, d):
    for blk in model.blocks:
        blk.scan_impl = "sequential"
        blk.connection_impl = "identity"
        blk.connection_damping = 1.0
        blk.phi_value_gate = torch.nn.Linear(3 * d, blk.r, bias=True)
        torch.nn.init.normal_(blk.phi_value_gate.weight, std=0.02)
        torch.nn.init.constant_(blk.phi_value_gate.bias, -2.0)
        blk.value_gate_input_mode = "current_prev_prefix"
        blk.couple_forget_to_value_gate = True
    model.prefix_condition_position = 1


@pytest.mark.parametrize("connection", ["identity", "cayley", "matrix_exp"])
def test_backbone_matches_reference_model(connection):
    affine_scan, model_mogt = _ref_modules()
    from mogt_b200.backbone import MOGTModel, configure_identity_coupled
    torch.manual_seed(0)
    d, r, layers, vocab = 64, 16, 2, 97
    ref = model_mogt.MOGTModel(vocab, d, layers, r)
    for p in ref.parameters():
        torch.nn.init.normal_(p, std=0.02)
    _configure_ref(ref, d)
    for blk in ref.blocks:
        blk.connection_impl = connection
        blk.connection_damping = 0.999 if connection != "identity" else 1.0

    def seq_scan(U, V, out_dtype):
        return affine_scan.affine_scan_sequential(U, V, state_dtype=torch.float32, output_dtype=out_dtype)

    mine = MOGTModel(vocab, d, layers, r, scan_fn=seq_scan)
    configure_identity_coupled(mine)
    for mb, rb in zip(mine.blocks, ref.blocks):
        mb.connection_impl = rb.connection_impl
        mb.connection_damping = rb.connection_damping
    missing = mine.load_state_dict(ref.state_dict(), strict=True)
    ids = torch.randint(0, vocab, (2, 40))
    with torch.no_grad():
        a = ref(ids)
        b = mine(ids)
    assert torch.allclose(a, b, rtol=1e-5, atol=1e-6), (a - b).abs().max()
