"""Tensor-level wrappers over the C ABI (no autograd).

Every function validates shapes the way the reference does (ValueError on bad
rank/shape, triton_scan.py:193-201), refuses CPU tensors (the reference's
Triton path raises the same way, triton_scan.py:191-192) and launches on the
current CUDA stream.  Nothing here computes on the CPU.  A device-side wait
that timed out in a call raises ``_native.DeviceTimeout`` from the next call
that uses the same workspace (at once with MOGT_SYNC_CHECK=1), or from
``mogt_b200.check_errors()``.
"""
from __future__ import annotations

import torch

from . import _native as N

__all__ = ["gated_scan_fwd", "gated_scan_bwd", "matrix_scan_fwd", "matrix_scan_bwd", "diag_scan_norm",
           "diag_scan_norm_bwd", "DiagScanNormFn",
           "affine_scan", "affine_grad_u", "gated_num_chunks"]


def _require_cuda(*ts, what):
    for t in ts:
        if t is not None and t.device.type != "cuda":
            raise ValueError(f"{what} requires CUDA tensors")


def gated_num_chunks(T: int, dk: int, dv: int, dtype: torch.dtype) -> int:
    return int(N.lib().mogt_gated_scan_num_chunks(T, dk, dv, N.dtype_code(dtype)))


def gated_scan_fwd(q, k, v, f, *, initial_state=None, output_dtype=None, want_final=False,
                   save_states=False, want_output=True, resume=False):
    """o_t = S_t^T q_t with S_t = f_t S_{t-1} + (1-f_t) k_t v_t^T.

    q, k: [B, H, T, dk]; v: [B, H, T, dv]; f: [B, H, T] (any float dtype, used
    as fp32).  bf16 inputs take the tensor-core path (dk = dv = 64); fp32
    inputs take the exact sequential path.  Returns (o, S_final, decay_final,
    chunk_states) with the optional members None unless requested;
    chunk_states [B, H, ceil(T/64), dk, dv] bf16 holds the state entering each
    64-step chunk (bf16 path only).

    resume=True (bf16 only): the previous call on this device and stream was a
    forward of the same k, v, f made without save_states (typically state-only,
    want_output=False); this call reuses its chunk-local states and runs only
    the carry from `initial_state` and the output pass
    (mogt_gated_scan_fwd_resume).
    """
    _require_cuda(q, k, v, f, initial_state, what="gated_scan")
    src_ptrs = (k.data_ptr(), v.data_ptr(), f.data_ptr())   # the caller's tensors, before any copy
    if k.ndim != 4 or v.ndim != 4 or f.ndim != 3 or (q is not None and q.ndim != 4):
        raise ValueError("q, k, v must be [B, H, T, d] and f must be [B, H, T]")
    B, H, T, dk = k.shape
    dv = v.shape[-1]
    if v.shape[:3] != (B, H, T) or f.shape != (B, H, T) or (q is not None and q.shape != k.shape):
        raise ValueError("q, k must be [B, H, T, dk], v [B, H, T, dv], f [B, H, T]")
    in_dtype = k.dtype
    if v.dtype != in_dtype or (q is not None and q.dtype != in_dtype):
        raise ValueError("q, k, v must share one dtype")
    if in_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("q, k, v must be bfloat16 or float32")
    out_dtype = output_dtype or in_dtype
    dev = k.device
    k = k.contiguous()
    v = v.contiguous()
    q = q.contiguous() if q is not None else None
    f = f.to(torch.float32).contiguous()
    BH = B * H
    o = torch.empty(B, H, T, dv, dtype=out_dtype, device=dev) if want_output else None
    S0 = None
    if initial_state is not None:
        if initial_state.shape != (B, H, dk, dv):
            raise ValueError("initial_state must be [B, H, dk, dv]")
        S0 = initial_state.to(torch.float32).contiguous()
    S_fin = torch.empty(B, H, dk, dv, dtype=torch.float32, device=dev) if want_final else None
    dec = torch.empty(B, H, dtype=torch.float32, device=dev) if want_final else None
    seg = None
    if save_states:
        nch = gated_num_chunks(T, dk, dv, in_dtype)
        if nch > 0:
            seg = torch.empty(B, H, nch, dk, dv, dtype=torch.bfloat16, device=dev)
    L = N.lib()
    icode, ocode = N.dtype_code(in_dtype), N.dtype_code(out_dtype)
    nbytes = L.mogt_gated_scan_fwd_workspace_bytes(BH, T, dk, dv, icode)
    with torch.cuda.device(dev):
        w = N.workspaces.entry(dev, nbytes, "gated_fwd")
        ws = w.buf
        if resume and in_dtype != torch.bfloat16:
            raise ValueError("resume needs bf16 inputs")
        # the chunk-local states a resumed call reuses are those of the last
        # forward on this workspace: same k, v, f, made without save_states
        tag = ("gated_fwd_local",) + src_ptrs + (BH, T, dk, dv)
        if resume and w.tag != tag:
            raise ValueError("resume=True needs the previous forward on this device and stream to be "
                             "a bf16 call with the same k, v, f made without save_states")
        fn = L.mogt_gated_scan_fwd_resume if resume else L.mogt_gated_scan_fwd
        name = "mogt_gated_scan_fwd_resume" if resume else "mogt_gated_scan_fwd"
        st = fn(N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(f), N.ptr(o), N.ptr(S0), N.ptr(S_fin), N.ptr(dec),
                N.ptr(seg), BH, T, dk, dv, icode, ocode, N.ptr(ws), ws.numel(), N.stream_ptr(dev))
        N.check(st, name)
        w.after_launch(name)
        w.tag = tag if (in_dtype == torch.bfloat16 and seg is None) else None
    return o, S_fin, dec, seg


def gated_scan_bwd(q, k, v, f, do, *, initial_state=None, want_dS0=False, chunk_states=None):
    """Gradients of sum(o * do) for o = gated_scan(q, k, v, f): returns
    (dq, dk, dv, df, dS0) with dq, dk, dv in the input dtype, df fp32 and dS0
    (gradient of the initial state) fp32 or None.

    float32 inputs: exact sequential kernels (any dk, dv <= 128).
    bfloat16 inputs (dk = dv = 64): the reverse-time chunked tensor-core
    kernel; `chunk_states` must be the per-chunk states returned by
    gated_scan_fwd(..., save_states=True) on the same inputs and initial state."""
    _require_cuda(q, k, v, f, do, initial_state, chunk_states, what="gated_scan backward")
    B, H, T, dk = k.shape
    dv = v.shape[-1]
    if q.shape != k.shape or v.shape[:3] != (B, H, T) or f.shape != (B, H, T) or do.shape != v.shape:
        raise ValueError("q, k: [B, H, T, dk]; v, do: [B, H, T, dv]; f: [B, H, T]")
    dt = k.dtype
    if dt not in (torch.float32, torch.bfloat16):
        raise ValueError("the gated-scan backward takes float32 or bfloat16 inputs")
    dev = k.device
    q, k, v, do = (t.to(dt).contiguous() for t in (q, k, v, do))
    f = f.to(torch.float32).contiguous()
    S0 = None
    cs = None
    if dt == torch.bfloat16:
        nch = gated_num_chunks(T, dk, dv, dt)
        if chunk_states is None or tuple(chunk_states.shape) != (B, H, nch, dk, dv) \
                or chunk_states.dtype != torch.bfloat16:
            raise ValueError("bfloat16 backward needs the forward's chunk_states "
                             f"[B, H, {nch}, {dk}, {dv}] bfloat16")
        cs = chunk_states.contiguous()
    else:
        S0 = None if initial_state is None else initial_state.to(torch.float32).contiguous()
    gq, gk = torch.empty_like(q), torch.empty_like(k)
    gv = torch.empty_like(v)
    gf = torch.empty(B, H, T, dtype=torch.float32, device=dev)
    gS0 = torch.empty(B, H, dk, dv, dtype=torch.float32, device=dev) if want_dS0 else None
    L = N.lib()
    code = N.dtype_code(dt)
    nbytes = L.mogt_gated_scan_bwd_workspace_bytes(B * H, T, dk, dv, code)
    with torch.cuda.device(dev):
        w = None
        if dt == torch.bfloat16:
            w = N.workspaces.entry(dev, nbytes, "gated_bwd")
            ws = w.buf
        else:
            ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        st = L.mogt_gated_scan_bwd(N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(f), N.ptr(do), N.ptr(S0),
                                   N.ptr(cs), N.ptr(gq), N.ptr(gk), N.ptr(gv), N.ptr(gf), N.ptr(gS0),
                                   B * H, T, dk, dv, code, N.ptr(ws), ws.numel(), N.stream_ptr(dev))
        N.check(st, "mogt_gated_scan_bwd")
        if w is not None:
            w.after_launch("mogt_gated_scan_bwd")
    return gq, gk, gv, gf, gS0


def matrix_scan_fwd(A, q, k, v, f, *, initial_state=None, output_dtype=None, want_final=False,
                    chunked=None, precision="fp32", save_for_backward=False):
    """o_t = S_t^T q_t with S_t = A_t S_{t-1} + (1-f_t) k_t v_t^T (dense A_t).
    A: [B, H, T, d, d]; q, k, v: [B, H, T, d]; f: [B, H, T]; d in {16, 32, 64}.
    Returns (o, S_final), or (o, S_final, saved) with save_for_backward.

    d = 64 (the default for T > 64, `chunked=None`) runs the chunked kernels:
    every 64-step chunk's transition prefix products and local state in
    parallel, the chunk carries composed per head, then the outputs per chunk.
    `precision="fp32"` (default) computes the chunks with fp32 FMAs;
    `"tf32x3"` on the tensor cores (bf16 q/k/v only), faster but with a bias
    that grows with T (4e-4 relative at T = 8192 for Cayley transitions).
    `chunked=False` forces the single sequential pass per head.
    `save_for_backward=True` (chunked only) also returns the forward's
    per-chunk states and products, which matrix_scan_bwd takes as `saved`."""
    _require_cuda(A, q, k, v, f, initial_state, what="matrix_scan")
    if A.ndim != 5 or q.ndim != 4:
        raise ValueError("A must be [B, H, T, d, d] and q, k, v [B, H, T, d]")
    B, H, T, d = q.shape
    if A.shape != (B, H, T, d, d) or k.shape != q.shape or v.shape != q.shape or f.shape != (B, H, T):
        raise ValueError("A: [B, H, T, d, d]; q, k, v: [B, H, T, d]; f: [B, H, T]")
    if q.dtype not in (torch.bfloat16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, v must share dtype bfloat16 or float32")
    if precision not in ("fp32", "tf32x3"):
        raise ValueError("precision must be 'fp32' or 'tf32x3'")
    out_dtype = output_dtype or q.dtype
    dev = q.device
    A = A.to(torch.float32).contiguous()
    q, k, v = (t.contiguous() for t in (q, k, v))
    f = f.to(torch.float32).contiguous()
    S0 = None if initial_state is None else initial_state.to(torch.float32).contiguous()
    o = torch.empty(B, H, T, d, dtype=out_dtype, device=dev)
    S_fin = torch.empty(B, H, d, d, dtype=torch.float32, device=dev) if want_final else None
    L = N.lib()
    icode, ocode = N.dtype_code(q.dtype), N.dtype_code(out_dtype)
    if chunked is None:
        chunked = d == 64 and (T > 64 or save_for_backward)
    if chunked and d != 64:
        raise ValueError("the chunked matrix scan supports d = 64 only")
    if save_for_backward and not chunked:
        raise ValueError("save_for_backward needs the chunked matrix scan (d = 64)")
    mode = N.MATRIX_TF32X3 if precision == "tf32x3" else N.MATRIX_FP32
    with torch.cuda.device(dev):
        if not chunked:
            st = L.mogt_matrix_scan_fwd(N.ptr(A), N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(f), N.ptr(o),
                                        N.ptr(S0), N.ptr(S_fin), B * H, T, d, icode, ocode,
                                        N.stream_ptr(dev))
            N.check(st, "mogt_matrix_scan_fwd")
            return o, S_fin
        nbytes = L.mogt_matrix_scan_chunked_scratch_bytes(B * H, T, d)
        scratch = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        w = N.workspaces.entry(dev, 256, "matrix_chunked")
        st = L.mogt_matrix_scan_fwd_chunked(N.ptr(A), N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(f), N.ptr(o),
                                            N.ptr(S0), N.ptr(S_fin), B * H, T, d, icode, ocode, mode,
                                            N.ptr(w.buf), N.ptr(scratch), nbytes, N.stream_ptr(dev))
        N.check(st, "mogt_matrix_scan_fwd_chunked")
        w.after_launch("mogt_matrix_scan_fwd_chunked")
    if save_for_backward:
        return o, S_fin, scratch
    return o, S_fin


def matrix_scan_bwd(A, q, k, v, f, do, saved, *, want_dS0=False):
    """Gradients of sum(o * do) for o = matrix_scan_fwd(A, q, k, v, f) (d = 64):
    returns (dA fp32, dq, dk, dv in the input dtype, df fp32, dS0 fp32 or
    None).  `saved` is the third result of matrix_scan_fwd(...,
    save_for_backward=True) on the same inputs (initial state included)."""
    _require_cuda(A, q, k, v, f, do, saved, what="matrix_scan backward")
    B, H, T, d = q.shape
    if A.shape != (B, H, T, d, d) or k.shape != q.shape or v.shape != q.shape or do.shape != q.shape \
            or f.shape != (B, H, T):
        raise ValueError("A: [B, H, T, d, d]; q, k, v, do: [B, H, T, d]; f: [B, H, T]")
    if d != 64:
        raise ValueError("the dense-transition backward supports d = 64")
    dt = q.dtype
    if dt not in (torch.bfloat16, torch.float32):
        raise ValueError("q, k, v must be bfloat16 or float32")
    dev = q.device
    A = A.to(torch.float32).contiguous()
    q, k, v, do = (t.to(dt).contiguous() for t in (q, k, v, do))
    f = f.to(torch.float32).contiguous()
    L = N.lib()
    if saved.numel() < L.mogt_matrix_scan_chunked_scratch_bytes(B * H, T, d):
        raise ValueError("`saved` is not the forward's saved state for these shapes")
    dA = torch.empty(B, H, T, d, d, dtype=torch.float32, device=dev)
    gq, gk, gv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    gf = torch.empty(B, H, T, dtype=torch.float32, device=dev)
    gS0 = torch.empty(B, H, d, d, dtype=torch.float32, device=dev) if want_dS0 else None
    nbytes = L.mogt_matrix_scan_bwd_scratch_bytes(B * H, T, d)
    with torch.cuda.device(dev):
        scratch = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        w = N.workspaces.entry(dev, 256, "matrix_bwd")
        st = L.mogt_matrix_scan_bwd(N.ptr(A), N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(f), N.ptr(do),
                                    N.ptr(saved), N.ptr(dA), N.ptr(gq), N.ptr(gk), N.ptr(gv), N.ptr(gf),
                                    N.ptr(gS0), B * H, T, d, N.dtype_code(dt), N.ptr(w.buf),
                                    N.ptr(scratch), nbytes, N.stream_ptr(dev))
        N.check(st, "mogt_matrix_scan_bwd")
        w.after_launch("mogt_matrix_scan_bwd")
    return dA, gq, gk, gv, gf, gS0


def diag_scan_norm(V, z, norm_weight, *, damping=1.0, eps=1e-6, initial_state=None,
                   output_dtype=None, want_final=False, return_scratch=False):
    """Fused identity-connection MOGT scan and RMSNorm readout:
    h_t = damping (1 - z_t[row]) h_{t-1} + V_t z_t[row] per channel (V times z
    rounded in V's dtype, as V * z.to(V.dtype) does), then per token
    y_t = h_t * rsqrt(mean(h_t^2) + eps) * norm_weight.
    V: [B, L, R, C] bf16/fp32; z: [B, L, R, 1] or [B, L, 1, 1] (or without
    the last axis) fp32 gates; norm_weight: [R*C].  Returns (y [B, L, R*C],
    H_final [B, R, C] fp32 or None)."""
    _require_cuda(V, z, norm_weight, initial_state, what="diag_scan_norm")
    if V.ndim != 4:
        raise ValueError("V must be [B, L, R, C]")
    B, L, R, C = V.shape
    zz = z.reshape(B, L, -1) if z.numel() in (B * L, B * L * R) else None
    if zz is None:
        raise ValueError("z must hold one gate per token or one per row")
    if V.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("V must be bfloat16 or float32")
    out_dtype = output_dtype or V.dtype
    dev = V.device
    V = V.contiguous()
    zz = zz.to(torch.float32).contiguous()
    w = norm_weight.to(torch.float32).contiguous()
    if w.numel() != R * C:
        raise ValueError("norm_weight must have R*C entries")
    H0 = None if initial_state is None else initial_state.to(torch.float32).contiguous()
    y = torch.empty(B, L, R * C, dtype=out_dtype, device=dev)
    Hf = torch.empty(B, R, C, dtype=torch.float32, device=dev) if want_final else None
    L_ = N.lib()
    nbytes = L_.mogt_diag_scan_norm_scratch_bytes(B, L, R, C, N.dtype_code(V.dtype))
    scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        wse = N.workspaces.entry(dev, 256, "diag_scan")
        status = wse.buf
        st = L_.mogt_diag_scan_norm_fwd(N.ptr(V), N.ptr(zz), zz.shape[-1], float(damping), N.ptr(H0),
                                        N.ptr(w), float(eps), N.ptr(y), N.ptr(Hf), B, L, R, C,
                                        N.dtype_code(V.dtype), N.dtype_code(out_dtype), N.ptr(status),
                                        N.ptr(scratch), scratch.numel(), N.stream_ptr(dev))
        N.check(st, "mogt_diag_scan_norm_fwd")
        wse.after_launch("mogt_diag_scan_norm_fwd")
    if return_scratch:
        return y, Hf, scratch
    return y, Hf


def diag_scan_norm_bwd(V, z, norm_weight, dy, fwd_scratch, *, damping=1.0, eps=1e-6, want_dH0=False):
    """Gradients of sum(y * dy) for y = diag_scan_norm(V, z, norm_weight, ...):
    returns (dV in V's dtype, dz fp32 shaped like z, d_norm_weight fp32,
    dH0 fp32 [B, R, C] or None).  `fwd_scratch` is the third result of
    diag_scan_norm(..., return_scratch=True) on the same inputs."""
    _require_cuda(V, z, norm_weight, dy, fwd_scratch, what="diag_scan_norm backward")
    B, L, R, C = V.shape
    zz = z.reshape(B, L, -1).to(torch.float32).contiguous()
    V = V.contiguous()
    dy = dy.reshape(B, L, R * C)
    if dy.dtype not in (torch.bfloat16, torch.float32):
        dy = dy.float()
    dy = dy.contiguous()
    w = norm_weight.to(torch.float32).contiguous()
    dev = V.device
    dV = torch.empty_like(V)
    dz = torch.empty(B, L, zz.shape[-1], dtype=torch.float32, device=dev)
    dw = torch.empty(R * C, dtype=torch.float32, device=dev)
    dH0 = torch.empty(B, R, C, dtype=torch.float32, device=dev) if want_dH0 else None
    L_ = N.lib()
    nbytes = L_.mogt_diag_scan_norm_bwd_scratch_bytes(B, L, R, C)
    with torch.cuda.device(dev):
        scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
        wse = N.workspaces.entry(dev, 256, "diag_bwd")
        st = L_.mogt_diag_scan_norm_bwd(N.ptr(V), N.ptr(zz), zz.shape[-1], float(damping), N.ptr(w), float(eps),
                                        N.ptr(dy), N.ptr(fwd_scratch), N.ptr(dV), N.ptr(dz), N.ptr(dw), N.ptr(dH0),
                                        B, L, R, C, N.dtype_code(V.dtype), N.dtype_code(dy.dtype),
                                        N.ptr(wse.buf), N.ptr(scratch), scratch.numel(), N.stream_ptr(dev))
        N.check(st, "mogt_diag_scan_norm_bwd")
        wse.after_launch("mogt_diag_scan_norm_bwd")
    return dV, dz.view(z.shape), dw.view(norm_weight.shape).to(norm_weight.dtype), dH0


class DiagScanNormFn(torch.autograd.Function):
    """Autograd for diag_scan_norm: the forward keeps its chunk carries for the
    reverse-time chunked backward (mogt_diag_scan_norm_bwd)."""

    @staticmethod
    def forward(ctx, V, z, norm_weight, initial_state, damping, eps, output_dtype):
        y, _, scratch = diag_scan_norm(V, z, norm_weight, damping=damping, eps=eps,
                                       initial_state=initial_state, output_dtype=output_dtype,
                                       return_scratch=True)
        ctx.save_for_backward(V, z, norm_weight, scratch)
        ctx.damping, ctx.eps = damping, eps
        ctx.has_h0 = initial_state is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        V, z, w, scratch = ctx.saved_tensors
        dV, dz, dw, dH0 = diag_scan_norm_bwd(V, z, w, dy, scratch, damping=ctx.damping, eps=ctx.eps,
                                             want_dH0=ctx.has_h0 and ctx.needs_input_grad[3])
        return dV, dz.to(z.dtype), dw, dH0, None, None, None


def _check_uv(U, V):
    if U.ndim != 4 or V.ndim != 4:
        raise ValueError("U and V must be rank-4 tensors")
    B, L, R, R2 = U.shape
    Bv, Lv, Rv, C = V.shape
    if (B, L, R) != (Bv, Lv, Rv) or R != R2:
        raise ValueError("U must be [B, L, R, R] and V must be [B, L, R, C]")
    return B, L, R, C


def affine_scan(U, V, *, output_dtype=torch.float32, return_prefix=False, reverse=False):
    """H_t = U_t H_{t-1} + V_t (fp32 state), optionally with the prefix products
    P_t = U_t ... U_0.  reverse=True computes the backward's adjoint
    Sigma_t = V_t + U_{t+1}^T Sigma_{t+1}.  V may be None for prefix-only."""
    _require_cuda(U, V, what="affine_scan")
    if V is None:
        if U.ndim != 4 or U.shape[-1] != U.shape[-2]:
            raise ValueError("U must be [B, L, R, R]")
        B, L, R, _ = U.shape
        C = 0
    else:
        B, L, R, C = _check_uv(U, V)
    if U.dtype not in (torch.float32, torch.bfloat16) or (V is not None and V.dtype not in (torch.float32, torch.bfloat16)):
        raise ValueError("U and V must be float32 or bfloat16")
    dev = U.device
    U = U.contiguous()
    V = V.contiguous() if V is not None else None
    H = torch.empty(B, L, R, C, dtype=output_dtype, device=dev) if C > 0 else None
    P = torch.empty(B, L, R, R, dtype=output_dtype, device=dev) if return_prefix else None
    Lb = N.lib()
    nbytes = Lb.mogt_affine_scan_workspace_bytes(B, L, R, C)
    with torch.cuda.device(dev):
        w = N.workspaces.entry(dev, nbytes, "affine")
        ws = w.buf
        st = Lb.mogt_affine_scan_fwd(N.ptr(U), N.ptr(V), N.ptr(H), N.ptr(P), B, L, R, C,
                                     N.dtype_code(U.dtype),
                                     N.dtype_code(V.dtype) if V is not None else N.dtype_code(U.dtype),
                                     N.dtype_code(output_dtype), int(reverse), N.ptr(ws), ws.numel(),
                                     N.stream_ptr(dev))
        N.check(st, "mogt_affine_scan_fwd")
        w.after_launch("mogt_affine_scan_fwd")
    return H, P


def affine_grad_u(sigma, H, *, output_dtype=torch.float32):
    """dU_t = Sigma_t H_{t-1}^T (H_{-1} = 0); sigma, H fp32 [B, L, R, C]."""
    _require_cuda(sigma, H, what="affine_grad_u")
    B, L, R, C = sigma.shape
    sigma = sigma.to(torch.float32).contiguous()
    H = H.to(torch.float32).contiguous()
    gU = torch.empty(B, L, R, R, dtype=output_dtype, device=sigma.device)
    with torch.cuda.device(sigma.device):
        st = N.lib().mogt_affine_grad_u(N.ptr(sigma), N.ptr(H), N.ptr(gU), B, L, R, C,
                                        N.dtype_code(output_dtype), N.stream_ptr(sigma.device))
    N.check(st, "mogt_affine_grad_u")
    return gU
