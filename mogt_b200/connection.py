"""Connection map of the MOGT block on the GPU, with autograd.

Replaces the reference's _build_transport (model_mogt.py:79-102): the
antisymmetrised phi_conn output A = (M - M^T) / r is mapped per token to the
transport U = damping * expm(A) ("matrix_exp") or damping * Cayley(A)
("cayley"), fp32 arithmetic, in one kernel launch (mogt_connection_map).

Backward:
  * expm: dL/dA is the Frechet derivative of expm at A^T applied to the
    upstream gradient, i.e. the upper-right block of expm([[A^T, G], [0, A^T]])
    (the block-triangular identity torch.matrix_exp's own backward uses); the
    2r x 2r exponentials run on the same kernel;
  * cayley: with S = A / 2 and U0 = (I - S)^{-1}(I + S),
    dL/dS = (I + S)^{-1} G (I + U0)^T  (since (I - S)^{-T} = (I + S)^{-1}).
  then dM = (dA - dA^T) / r.
"""
from __future__ import annotations

import torch

from . import _native as N

__all__ = ["connection_map", "ConnectionMapFn"]

_MODES = {"matrix_exp": 0, "cayley": 1}


def _launch(M, n, mode, skew, scale, damping, out_dtype):
    if M.device.type != "cuda":
        raise ValueError("connection_map requires CUDA tensors")
    M = M.contiguous()
    U = torch.empty(M.shape, dtype=out_dtype, device=M.device)
    count = M.numel() // (n * n)
    with torch.cuda.device(M.device):
        st = N.lib().mogt_connection_map(N.ptr(M), N.ptr(U), count, n, mode, int(skew), float(scale),
                                         float(damping), N.dtype_code(M.dtype), N.dtype_code(out_dtype),
                                         N.stream_ptr(M.device))
    N.check(st, "mogt_connection_map")
    return U


class ConnectionMapFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, M, impl, damping, out_dtype):
        n = M.shape[-1]
        U = _launch(M, n, _MODES[impl], True, 1.0 / n, damping, out_dtype)
        ctx.save_for_backward(M)
        ctx.impl, ctx.damping = impl, damping
        return U

    @staticmethod
    def backward(ctx, gU):
        (M,) = ctx.saved_tensors
        n = M.shape[-1]
        lead = M.shape[:-2]
        A = (M - M.transpose(-1, -2)).to(M.dtype).float() / n
        G = gU.float() * ctx.damping
        A = A.reshape(-1, n, n)
        G = G.reshape(-1, n, n)
        At = A.transpose(-1, -2)
        if ctx.impl == "matrix_exp":
            blk = torch.zeros(A.shape[0], 2 * n, 2 * n, dtype=torch.float32, device=A.device)
            blk[:, :n, :n] = At
            blk[:, n:, n:] = At
            blk[:, :n, n:] = G
            E = _launch(blk, 2 * n, 0, False, 1.0, 1.0, torch.float32)
            dA = E[:, :n, n:]
        else:
            eye = torch.eye(n, dtype=torch.float32, device=A.device)
            S = 0.5 * A
            U0 = torch.linalg.solve(eye - S, eye + S)
            dS = torch.linalg.solve(eye + S, G @ (eye + U0).transpose(-1, -2))
            dA = 0.5 * dS
        dM = (dA - dA.transpose(-1, -2)) / n
        return dM.reshape(lead + (n, n)).to(M.dtype), None, None, None


def connection_map(M, impl="matrix_exp", damping=0.999, output_dtype=None):
    """M: [..., r, r] phi_conn output (any float dtype, CUDA).  Returns
    damping * map((M - M^T) / r) in ``output_dtype`` (default M's dtype);
    impl "matrix_exp" or "cayley" (model_mogt.py:79-102)."""
    if impl not in _MODES:
        raise ValueError(f"unsupported connection_impl: {impl}")
    if M.shape[-1] != M.shape[-2] or M.shape[-1] not in (8, 16):
        raise ValueError("connection_map takes [..., r, r] with r in {8, 16}")
    out_dtype = output_dtype or M.dtype
    if torch.is_grad_enabled() and M.requires_grad:
        return ConnectionMapFn.apply(M, impl, float(damping), out_dtype)
    return _launch(M, M.shape[-1], _MODES[impl], True, 1.0 / M.shape[-1], float(damping), out_dtype)
