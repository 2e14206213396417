"""mogt_b200 — B200-native (sm_100a) implementation of MOGT's scan operator.

Public API:
  * ``mogt_b200.triton_scan``: drop-in for the reference module of the same
    name (triton_affine_scan_hybrid, triton_affine_local_scan,
    triton_fused_scan, _TritonAffineScanHybridAutograd);
  * ``gated_scan(q, k, v, f)``: the headed, gated form with autograd;
  * ``matrix_scan(A, q, k, v, f)``: the dense-transition form with autograd;
  * ``check_errors()``: raise if a kernel recorded a device-side timeout;
  * ``ops``: the tensor-level wrappers of the C ABI (include/mogt_scan.h).
"""
from . import ops, triton_scan  # noqa: F401
from .gated import gated_scan  # noqa: F401
from .matrix import matrix_scan  # noqa: F401
from ._native import check_errors  # noqa: F401


__all__ = ["gated_scan", "matrix_scan", "check_errors", "ops", "triton_scan", "install_as_triton_scan"]


def install_as_triton_scan():
    """Register ``mogt_b200.triton_scan`` as the top-level module
    ``triton_scan`` so the reference model's lazy ``from triton_scan import
    ...`` (model_mogt.py:190, 195) resolves to this implementation."""
    import sys
    sys.modules["triton_scan"] = triton_scan
    return triton_scan
