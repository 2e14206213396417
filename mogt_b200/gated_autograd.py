"""torch.autograd.Function for the headed gated scan.

The forward saves only its inputs (like the reference's
_TritonAffineScanHybridAutograd, triton_scan.py:314-356) and the backward
recomputes what it needs inside libmogt_scan.so.
"""
from __future__ import annotations

import torch

from . import ops


class GatedScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, f, output_dtype, initial_state):
        with torch.autograd.profiler.record_function("mogt.gated_scan.forward"):
            o, _, _, _ = ops.gated_scan_fwd(q, k, v, f, initial_state=initial_state,
                                            output_dtype=output_dtype)
        ctx.save_for_backward(q, k, v, f, initial_state)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, f, S0 = ctx.saved_tensors
        with torch.autograd.profiler.record_function("mogt.gated_scan.backward"):
            dt = k.dtype
            # the exact fp32 sequential kernels serve every input dtype
            cast = (lambda t: t.float()) if dt != torch.float32 else (lambda t: t)
            dq, dk, dv, df, dS0 = ops.gated_scan_bwd(
                cast(q), cast(k), cast(v), f, cast(do), initial_state=S0,
                want_dS0=S0 is not None and ctx.needs_input_grad[5])
            dq, dk, dv = dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)
        return dq, dk, dv, df.to(f.dtype), None, dS0
