"""CPU checks of the C ABI: the library loads and exports every symbol that
include/*.h declares, and the ctypes signature table covers them all."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"\b(mogt_[a-z0-9_]+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"mogt_gated_scan_fwd", "mogt_affine_scan_fwd", "mogt_affine_grad_u"} <= names


def test_library_exports_every_declared_symbol():
    from mogt_b200 import _native
    lib = _native.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert declared_symbols() == set(_native.SIGNATURES), "ctypes table out of sync with the header"
    assert lib.mogt_abi_version() == 2
    assert lib.mogt_status_string(5) == b"device-side wait timed out"


def test_workspace_sizes_without_gpu():
    from mogt_b200 import _native
    lib = _native.lib()
    assert lib.mogt_gated_scan_num_chunks(32768, 64, 64, _native.BF16) == 512
    assert lib.mogt_gated_scan_num_chunks(32768, 64, 64, _native.F32) == 0
    ws = lib.mogt_gated_scan_fwd_workspace_bytes(12, 32768, 64, 64, _native.BF16)
    assert ws >= 12 * 2 * 64 * 64 * 4  # at least one stripe state pair per head
    assert lib.mogt_affine_scan_workspace_bytes(1, 32768, 16, 48) > 0


def test_cpu_tensors_are_refused():
    import torch
    import mogt_b200
    q = torch.zeros(1, 1, 4, 64, dtype=torch.bfloat16)
    f = torch.ones(1, 1, 4)
    with pytest.raises(ValueError, match="CUDA"):
        mogt_b200.gated_scan(q, q, q, f)
    with pytest.raises(ValueError, match="CUDA"):
        mogt_b200.triton_scan.triton_affine_scan_hybrid(torch.zeros(1, 4, 16, 16), torch.zeros(1, 4, 16, 48))
    with pytest.raises(ValueError):
        mogt_b200.triton_scan.triton_affine_scan_hybrid(torch.zeros(1, 4, 16, 16), torch.zeros(1, 4, 16, 48),
                                                        carry_scan="nope")
