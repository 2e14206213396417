"""Drop-in replacement for the reference's ``triton_scan`` module.

Same public names, signatures, return conventions and errors as lkcfqy/MOGT
``triton_scan.py``, backed by libmogt_scan.so (hand-written sm_100a CUDA)
instead of Triton kernels plus a Python carry loop.  ``model_mogt.py``
imports these names lazily (model_mogt.py:190, 195); putting this module on
the import path as ``triton_scan`` (or registering it in ``sys.modules``, see
``mogt_b200.install_as_triton_scan``) makes the reference model call it
unchanged.

``block_size``, ``block_c`` and ``carry_scan`` are accepted and validated like
the reference; the single-launch kernel does not need them (its carry scan is
an in-kernel decoupled look-back), except that ``triton_affine_local_scan``
honours ``block_size`` because its outputs are defined per block.
"""
from __future__ import annotations

import torch

from . import ops

__all__ = [
    "triton_fused_scan",
    "triton_affine_local_scan",
    "triton_affine_scan_hybrid",
    "_TritonAffineScanHybridAutograd",
    "_triton_affine_scan_hybrid_forward",
    "_triton_affine_scan_hybrid_backward",
]


def _next_power_of_two(value: int) -> int:
    # triton_scan.py:8-11
    if value <= 0:
        raise ValueError("value must be positive")
    return 1 << (value - 1).bit_length()


def triton_fused_scan(U: torch.Tensor):
    """Y_t = U_t @ Y_{t-1}, Y_0 = I: prefix products only (triton_scan.py:151-175).
    Returns a tensor like U."""
    B, L, R, _R = U.shape
    assert R == _R, "the last two dimensions must be square"
    _, Y = ops.affine_scan(U, None, output_dtype=U.dtype, return_prefix=True)
    return Y


def triton_affine_local_scan(U: torch.Tensor, V: torch.Tensor, *, block_size: int = 256,
                             block_c: int = 32):
    """Block-local affine prefixes and per-block summaries (triton_scan.py:178-229).

    Returns (U_prefix, H_prefix, U_summary, H_summary), all fp32, where the
    prefixes restart from (I, 0) at every block of ``block_size`` steps."""
    if U.device.type != "cuda" or V.device.type != "cuda":
        raise ValueError("triton_affine_local_scan requires CUDA tensors")
    if U.ndim != 4 or V.ndim != 4:
        raise ValueError("U and V must be rank-4 tensors")
    B, L, R, R2 = U.shape
    Bv, Lv, Rv, C = V.shape
    if (B, L, R) != (Bv, Lv, Rv) or R != R2:
        raise ValueError("U must be [B, L, R, R] and V must be [B, L, R, C]")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    _next_power_of_two(block_c)
    nb = (L + block_size - 1) // block_size
    Lp = nb * block_size
    Uw, Vw = U, V
    if Lp != L:
        # identity / zero steps leave a block's prefix unchanged past L
        eye = torch.eye(R, device=U.device, dtype=U.dtype).expand(B, Lp - L, R, R)
        Uw = torch.cat([U, eye], 1)
        Vw = torch.cat([V, V.new_zeros(B, Lp - L, R, C)], 1)
    H, P = ops.affine_scan(Uw.reshape(B * nb, block_size, R, R), Vw.reshape(B * nb, block_size, R, C),
                           output_dtype=torch.float32, return_prefix=True)
    H = H.view(B, nb, block_size, R, C)
    P = P.view(B, nb, block_size, R, R)
    U_summary = P[:, :, -1].contiguous()
    H_summary = H[:, :, -1].contiguous()
    U_prefix = P.reshape(B, Lp, R, R)[:, :L]
    H_prefix = H.reshape(B, Lp, R, C)[:, :L]
    return U_prefix, H_prefix, U_summary, H_summary


def _triton_affine_scan_hybrid_forward(U, V, *, block_size=256, block_c=32, carry_scan="sequential",
                                       output_dtype=None, return_prefix=False):
    """Full affine scan H_t = U_t H_{t-1} + V_t (triton_scan.py:232-311), one launch."""
    if carry_scan not in {"sequential", "doubling"}:
        raise ValueError("carry_scan must be 'sequential' or 'doubling'")
    if U.device.type != "cuda" or V.device.type != "cuda":
        raise ValueError("triton_affine_local_scan requires CUDA tensors")
    output_dtype = output_dtype or V.dtype
    with torch.autograd.profiler.record_function("triton_hybrid.local_scan"):
        H, P = ops.affine_scan(U, V, output_dtype=output_dtype, return_prefix=return_prefix)
    if not return_prefix:
        return H
    return P, H


class _TritonAffineScanHybridAutograd(torch.autograd.Function):
    """Same contract as triton_scan.py:314-356: saves (U, V) only and
    recomputes in backward."""

    @staticmethod
    def forward(ctx, U, V, block_size, block_c, carry_scan, output_dtype):
        with torch.autograd.profiler.record_function("triton_hybrid.forward"):
            ctx.block_size = block_size
            ctx.block_c = block_c
            ctx.carry_scan = carry_scan
            ctx.output_dtype = output_dtype or V.dtype
            ctx.save_for_backward(U, V)
            return _triton_affine_scan_hybrid_forward(U, V, block_size=block_size, block_c=block_c,
                                                      carry_scan=carry_scan,
                                                      output_dtype=ctx.output_dtype,
                                                      return_prefix=False)

    @staticmethod
    def backward(ctx, grad_output):
        U_saved, V_saved = ctx.saved_tensors
        with torch.autograd.profiler.record_function("triton_hybrid.backward_recompute"):
            grad_u, grad_v = _triton_affine_scan_hybrid_backward(
                U_saved, V_saved, grad_output, block_size=ctx.block_size, block_c=ctx.block_c,
                carry_scan=ctx.carry_scan, need_grad_u=ctx.needs_input_grad[0],
                need_grad_v=ctx.needs_input_grad[1])
        return grad_u, grad_v, None, None, None, None


def _triton_affine_scan_hybrid_backward(U, V, grad_H, *, block_size, block_c, carry_scan,
                                        need_grad_u, need_grad_v):
    """Reverse scan Sigma_t = g_t + U_{t+1}^T Sigma_{t+1}; dV = Sigma,
    dU_t = Sigma_t H_{t-1}^T (triton_scan.py:359-426, affine_scan.py:65-124)."""
    if U.device.type != "cuda":
        raise ValueError("the MOGT scan backward requires CUDA tensors")
    g = grad_H if grad_H.dtype in (torch.float32, torch.bfloat16) else grad_H.float()
    H_prefix = None
    if need_grad_u:
        with torch.autograd.profiler.record_function("affine_backward.recompute_prefix_hybrid"):
            H_prefix, _ = ops.affine_scan(U, V, output_dtype=torch.float32)
    with torch.autograd.profiler.record_function("affine_backward.reverse_scan_hybrid"):
        sigma, _ = ops.affine_scan(U, g, output_dtype=torch.float32, reverse=True)
    grad_v = sigma.to(V.dtype) if need_grad_v else None
    grad_u = None
    if need_grad_u:
        with torch.autograd.profiler.record_function("affine_backward.grad_u_matmul"):
            grad_u = ops.affine_grad_u(sigma, H_prefix, output_dtype=torch.float32).to(U.dtype)
    return grad_u, grad_v


def triton_affine_scan_hybrid(U, V, *, block_size: int = 256, block_c: int = 32,
                              carry_scan: str = "sequential", output_dtype=None,
                              return_prefix: bool = False):
    """Public entry (triton_scan.py:429-477)."""
    if return_prefix:
        return _triton_affine_scan_hybrid_forward(U, V, block_size=block_size, block_c=block_c,
                                                  carry_scan=carry_scan, output_dtype=output_dtype,
                                                  return_prefix=True)
    needs_grad = torch.is_grad_enabled() and (U.requires_grad or V.requires_grad)
    if needs_grad:
        return _TritonAffineScanHybridAutograd.apply(U, V, block_size, block_c, carry_scan,
                                                     output_dtype)
    return _triton_affine_scan_hybrid_forward(U, V, block_size=block_size, block_c=block_c,
                                              carry_scan=carry_scan, output_dtype=output_dtype,
                                              return_prefix=False)
