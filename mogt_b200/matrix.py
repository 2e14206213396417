"""Dense-transition headed scan with autograd:  o = matrix_scan(A, q, k, v, f).

    S_t = A_t S_{t-1} + (1 - f_t) k_t v_t^T,   o_t = S_t^T q_t

This is the reference operator (affine_scan.py:14-62 with U_t = A_t,
V_t = (1 - f_t) k_t v_t^T) followed by the readout einsum.  Like the
reference's _TritonAffineScanHybridAutograd (triton_scan.py:314-356) the
forward saves its inputs; it also keeps the chunked forward's per-chunk
entering states and transition products, which the reverse-time chunked
backward (affine_scan.py:65-124 in chunked form) reads instead of recomputing
the forward carries.
"""
from __future__ import annotations

import torch

from . import ops

__all__ = ["matrix_scan", "MatrixScanFn"]


class MatrixScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A, q, k, v, f, initial_state, output_dtype, precision):
        with torch.autograd.profiler.record_function("mogt.matrix_scan.forward"):
            o, _, saved = ops.matrix_scan_fwd(A, q, k, v, f, initial_state=initial_state,
                                              output_dtype=output_dtype, precision=precision,
                                              save_for_backward=True)
        ctx.save_for_backward(A, q, k, v, f, saved)
        ctx.has_S0 = initial_state is not None
        return o

    @staticmethod
    def backward(ctx, do):
        A, q, k, v, f, saved = ctx.saved_tensors
        want_dS0 = ctx.has_S0 and ctx.needs_input_grad[5]
        with torch.autograd.profiler.record_function("mogt.matrix_scan.backward"):
            dA, dq, dk, dv, df, dS0 = ops.matrix_scan_bwd(A, q, k, v, f, do.to(q.dtype), saved,
                                                          want_dS0=want_dS0)
        return dA.to(A.dtype), dq, dk, dv, df.to(f.dtype), dS0, None, None


def matrix_scan(A, q, k, v, f, *, initial_state=None, output_dtype=None, precision="fp32"):
    """A: [B, H, T, d, d] fp32 transitions; q, k, v: [B, H, T, d] (bf16 or
    fp32); f: [B, H, T] gates.  Returns o: [B, H, T, d] in ``output_dtype``
    (default: q's dtype).  Differentiable in A, q, k, v, f and the initial
    state when d = 64 (the chunked kernels); ``precision`` as in
    ops.matrix_scan_fwd."""
    needs_grad = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (A, q, k, v, f, initial_state))
    if needs_grad:
        return MatrixScanFn.apply(A, q, k, v, f, initial_state, output_dtype, precision)
    with torch.autograd.profiler.record_function("mogt.matrix_scan"):
        o, _ = ops.matrix_scan_fwd(A, q, k, v, f, initial_state=initial_state,
                                   output_dtype=output_dtype, precision=precision)
    return o
