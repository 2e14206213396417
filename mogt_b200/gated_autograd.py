"""torch.autograd.Function for the headed gated scan.

Like the reference's _TritonAffineScanHybridAutograd (triton_scan.py:
314-356) the forward saves its inputs; on the bf16 64x64 path it also keeps
the bf16 state entering every 64-step chunk, which the reverse-time chunked
backward reads instead of recomputing the forward.
"""
from __future__ import annotations

import torch

from . import ops


class GatedScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, f, output_dtype, initial_state):
        tc = k.dtype == torch.bfloat16 and k.shape[-1] == 64 and v.shape[-1] == 64
        with torch.autograd.profiler.record_function("mogt.gated_scan.forward"):
            o, _, _, cs = ops.gated_scan_fwd(q, k, v, f, initial_state=initial_state,
                                             output_dtype=output_dtype, save_states=tc)
        ctx.tc = tc and cs is not None
        ctx.save_for_backward(q, k, v, f, initial_state, cs if ctx.tc else None)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, f, S0, cs = ctx.saved_tensors
        want_dS0 = S0 is not None and ctx.needs_input_grad[5]
        with torch.autograd.profiler.record_function("mogt.gated_scan.backward"):
            if ctx.tc:
                # reverse-time chunked tensor-core kernel on the forward's chunk states
                dq, dk, dv, df, dS0 = ops.gated_scan_bwd(q, k, v, f, do.to(k.dtype), chunk_states=cs,
                                                         want_dS0=want_dS0)
            else:
                # exact fp32 sequential kernels for every other shape and dtype
                dt = k.dtype
                cast = (lambda t: t.float()) if dt != torch.float32 else (lambda t: t)
                dq, dk, dv, df, dS0 = ops.gated_scan_bwd(
                    cast(q), cast(k), cast(v), f, cast(do), initial_state=S0, want_dS0=want_dS0)
            dq, dk, dv = dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)
        return dq, dk, dv, df.to(f.dtype), None, dS0
