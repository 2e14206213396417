"""Headed gated scan with autograd:  o = gated_scan(q, k, v, f).

    S_t = f_t S_{t-1} + (1 - f_t) k_t v_t^T,   o_t = S_t^T q_t

This is the reference operator (affine_scan.py:14-62 with U_t = f_t I,
V_t = (1 - f_t) k_t v_t^T) followed by the readout einsum, evaluated by the
chunked tensor-core kernel for bf16 inputs and by the exact sequential kernel
for fp32 inputs.
"""
from __future__ import annotations

import torch

from . import ops

__all__ = ["gated_scan"]


def gated_scan(q, k, v, f, *, output_dtype=None, initial_state=None):
    """q, k: [B, H, T, dk]; v: [B, H, T, dv]; f: [B, H, T] gates in [0, 1].
    Returns o: [B, H, T, dv] in ``output_dtype`` (default: the input dtype)."""
    needs_grad = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (q, k, v, f, initial_state))
    if needs_grad:
        from .gated_autograd import GatedScanFn
        return GatedScanFn.apply(q, k, v, f, output_dtype, initial_state)
    with torch.autograd.profiler.record_function("mogt.gated_scan"):
        o, _, _, _ = ops.gated_scan_fwd(q, k, v, f, initial_state=initial_state,
                                        output_dtype=output_dtype)
    return o
