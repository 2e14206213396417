"""Wiring of the reference's hybrid model to the drop-in (model_hybrid.py:
117-147 configure_mogt, model_mogt.py:185-203 scan dispatch), on the CPU.

The reference tree is imported read-only from MOGT_REFERENCE_DIR (the test
is skipped where it is absent).  After mogt_b200.install_as_triton_scan(),
the reference HybridBackbone configured with configure_mogt(scan_impl=
"triton_hybrid") resolves its lazy `from triton_scan import ...` to this
package: on CPU tensors the drop-in refuses with its own error (no CPU
fallback), and with the drop-in's entry point observed, one training step
runs through it with the kwargs configure_mogt set."""
import os
import sys
from pathlib import Path

import pytest
import torch

REF = Path(os.environ["MOGT_REFERENCE_DIR"]) if os.environ.get("MOGT_REFERENCE_DIR") else None
pytestmark = pytest.mark.skipif(REF is None or not (REF / "model_hybrid.py").exists(),
                                reason="reference tree absent (set MOGT_REFERENCE_DIR)")


def _hybrid():
    sys.dont_write_bytecode = True
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import model_hybrid
    torch.manual_seed(0)
    m = model_hybrid.HybridBackbone(vocab_size=50, d_model=64, num_layers=2, num_heads=4, r=16,
                                    pattern="alternating")
    m.configure_mogt(scan_impl="triton_hybrid", connection_impl="cayley", scan_block_size=128)
    return m


def test_reference_hybrid_reaches_the_drop_in():
    import mogt_b200
    saved = sys.modules.get("triton_scan")
    try:
        mogt_b200.install_as_triton_scan()
        m = _hybrid()
        ids = torch.randint(0, 50, (1, 24))
        with pytest.raises(ValueError, match="CUDA"):
            m(ids)
    finally:
        if saved is not None:
            sys.modules["triton_scan"] = saved
        else:
            sys.modules.pop("triton_scan", None)


def test_training_step_through_the_drop_in_entry(monkeypatch):
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import affine_scan  # the reference's sequential scan
    import mogt_b200
    calls = []

    def observed(U, V, *, block_size=256, block_c=32, carry_scan="sequential", output_dtype=None,
                 return_prefix=False):
        calls.append(dict(block_size=block_size, block_c=block_c, carry_scan=carry_scan,
                          output_dtype=output_dtype, shape=tuple(V.shape)))
        return affine_scan.affine_scan_sequential(U, V, output_dtype=output_dtype)

    monkeypatch.setattr(mogt_b200.triton_scan, "triton_affine_scan_hybrid", observed)
    saved = sys.modules.get("triton_scan")
    try:
        mogt_b200.install_as_triton_scan()
        m = _hybrid()
        ids = torch.randint(0, 50, (2, 24))
        out = m(ids)
        loss = out.float().pow(2).mean() if torch.is_tensor(out) else out[0].float().pow(2).mean()
        loss.backward()
    finally:
        if saved is not None:
            sys.modules["triton_scan"] = saved
        else:
            sys.modules.pop("triton_scan", None)
    assert calls and all(c["block_size"] == 128 and c["carry_scan"] == "sequential" for c in calls)
    assert all(c["shape"][-2] == 16 for c in calls)
