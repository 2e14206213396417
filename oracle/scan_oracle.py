"""CPU oracle for MOGT's affine / gated scan — TEST INFRASTRUCTURE ONLY.

This module is a numpy restatement of the reference's PyTorch scan algorithm
(lkcfqy/MOGT ``affine_scan.py``).  It exists to check the CUDA product path;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import it.  Nothing in ``mogt_b200`` imports it and the
product path never falls back to it.

Parity pin: every function here is checked (``tests/test_oracle.py``) against
golden vectors that ``tests/golden/make_golden.py`` produced by running the
reference's own ``affine_scan.py`` functions in the build container, and
against the algebraic identities of the reference's sanity script
(``sanity_affine_scan.py:19-61, 102-135``, tolerance 1e-10 in float64).

Conventions (identical to the reference):
  U : [B, L, R, R]   transition,   V : [B, L, R, C]   input
  H_t = U_t @ H_{t-1} + V_t,  H_0 = 0 (H_{-1} = 0 before the first step)
Headed form (BASELINE configs 1/2/3/5), B*H folded into the batch:
  S_t = f_t * S_{t-1} + (1 - f_t) * k_t v_t^T,   o_t = S_t^T q_t
which is the affine recurrence with U_t = f_t * I and V_t = (1-f_t) k_t v_t^T.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "affine_combine",
    "affine_scan_sequential",
    "affine_scan_sequential_backward",
    "affine_scan_doubling",
    "affine_scan_block_reference",
    "gated_scan_dense",
    "gated_scan",
    "gated_scan_backward",
    "matrix_scan",
    "matrix_scan_backward",
    "matrix_scan_stream",
    "matrix_scan_backward_stream",
]


def _check_uv(U, V):
    # affine_scan.py:26-32 — same ValueError conditions.
    if U.ndim != 4 or V.ndim != 4:
        raise ValueError("U and V must be rank-4 tensors")
    B, L, R, R2 = U.shape
    Bv, Lv, Rv, C = V.shape
    if (B, L, R) != (Bv, Lv, Rv) or R != R2:
        raise ValueError("U must be [B, L, R, R] and V must be [B, L, R, C]")
    return B, L, R, C


def affine_combine(U_next, V_next, U_prev, V_prev):
    """(U2,V2) o (U1,V1) = (U2 U1, U2 V1 + V2).  affine_scan.py:4-11."""
    return U_next @ U_prev, U_next @ V_prev + V_next


def affine_scan_sequential(U, V, *, state_dtype=np.float64, output_dtype=None,
                           return_prefix=False):
    """T-step loop of batched matmuls.  affine_scan.py:14-62.

    ``output_dtype`` defaults to V's dtype (affine_scan.py:34).  Each step is
    ``H = U_t @ H + V_t`` in ``state_dtype`` (affine_scan.py:48-51); the
    optional prefix product is ``P = U_t @ P`` starting from I (:43-55).
    """
    B, L, R, C = _check_uv(U, V)
    output_dtype = output_dtype or V.dtype
    Uw = U.astype(state_dtype, copy=False)
    Vw = V.astype(state_dtype, copy=False)
    H = np.zeros((B, R, C), dtype=state_dtype)
    Hs = np.empty((B, L, R, C), dtype=output_dtype)
    Ps = None
    if return_prefix:
        P = np.broadcast_to(np.eye(R, dtype=state_dtype), (B, R, R)).copy()
        Ps = np.empty((B, L, R, R), dtype=output_dtype)
    for t in range(L):
        Ut = Uw[:, t]
        H = np.matmul(Ut, H) + Vw[:, t]
        Hs[:, t] = H
        if return_prefix:
            P = np.matmul(Ut, P)
            Ps[:, t] = P
    if not return_prefix:
        return Hs
    return Ps, Hs


def affine_scan_sequential_backward(U, V, grad_H, *, state_dtype=np.float64,
                                    need_grad_u=True, need_grad_v=True):
    """Recompute-then-reverse-scan backward.  affine_scan.py:65-124.

    Sigma_t = g_t + U_{t+1}^T Sigma_{t+1};  dV_t = Sigma_t;
    dU_t = Sigma_t H_{t-1}^T  (affine_scan.py:111-118).
    """
    B, L, R, C = _check_uv(U, V)
    if grad_H.shape != (B, L, R, C):
        raise ValueError("grad_H must match V shape [B, L, R, C]")
    Uw = U.astype(state_dtype, copy=False)
    Vw = V.astype(state_dtype, copy=False)
    gw = grad_H.astype(state_dtype, copy=False)
    H_prev_states = []
    H = np.zeros((B, R, C), dtype=state_dtype)
    for t in range(L):  # affine_scan.py:101-105
        if need_grad_u:
            H_prev_states.append(H)
        H = np.matmul(Uw[:, t], H) + Vw[:, t]
    gU = np.empty_like(Uw) if need_grad_u else None
    gV = np.empty_like(Vw) if need_grad_v else None
    carry = np.zeros((B, R, C), dtype=state_dtype)
    for t in range(L - 1, -1, -1):  # affine_scan.py:111-118
        tot = gw[:, t] + carry
        if need_grad_v:
            gV[:, t] = tot
        if need_grad_u:
            gU[:, t] = np.matmul(tot, np.swapaxes(H_prev_states[t], -1, -2))
        carry = np.matmul(np.swapaxes(Uw[:, t], -1, -2), tot)
    if gU is not None:
        gU = gU.astype(U.dtype)
    if gV is not None:
        gV = gV.astype(V.dtype)
    return gU, gV


def affine_scan_doubling(U, V, *, state_dtype=np.float64, output_dtype=None,
                         return_prefix=False):
    """Hillis-Steele inclusive scan, log2(L) passes.  affine_scan.py:127-172."""
    B, L, R, C = _check_uv(U, V)
    output_dtype = output_dtype or V.dtype
    P = U.astype(state_dtype).copy()
    H = V.astype(state_dtype).copy()
    off = 1
    while off < L:
        Pp, Hp = P.copy(), H.copy()
        P[:, off:] = np.matmul(Pp[:, off:], Pp[:, :-off])
        H[:, off:] = np.matmul(Pp[:, off:], Hp[:, :-off]) + Hp[:, off:]
        off *= 2
    if not return_prefix:
        return H.astype(output_dtype)
    return P.astype(output_dtype), H.astype(output_dtype)


def affine_scan_block_reference(U, V, *, block_size=256, state_dtype=np.float64,
                                output_dtype=None, carry_scan="sequential",
                                return_prefix=False):
    """Block-local scan + summary scan + carry apply.  affine_scan.py:175-278."""
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    if carry_scan not in {"sequential", "doubling"}:
        raise ValueError("carry_scan must be 'sequential' or 'doubling'")
    B, L, R, C = _check_uv(U, V)
    output_dtype = output_dtype or V.dtype
    nb = (L + block_size - 1) // block_size
    loc_P, loc_H, sumP, sumH, ranges = [], [], [], [], []
    for b in range(nb):
        s, e = b * block_size, min((b + 1) * block_size, L)
        ranges.append((s, e))
        Pl, Hl = affine_scan_sequential(U[:, s:e], V[:, s:e], state_dtype=state_dtype,
                                        output_dtype=state_dtype, return_prefix=True)
        loc_P.append(Pl)
        loc_H.append(Hl)
        sumP.append(Pl[:, -1])
        sumH.append(Hl[:, -1])
    bP, bH = np.stack(sumP, 1), np.stack(sumH, 1)
    scan = affine_scan_sequential if carry_scan == "sequential" else affine_scan_doubling
    incP, incH = scan(bP, bH, state_dtype=state_dtype, output_dtype=state_dtype,
                      return_prefix=True)
    cP = np.broadcast_to(np.eye(R, dtype=state_dtype), (B, nb, R, R)).copy()
    cH = np.zeros((B, nb, R, C), dtype=state_dtype)
    if nb > 1:
        cP[:, 1:] = incP[:, :-1]
        cH[:, 1:] = incH[:, :-1]
    outP, outH = [], []
    for b, (s, e) in enumerate(ranges):
        outP.append(np.matmul(loc_P[b], cP[:, b][:, None]))
        outH.append(np.matmul(loc_P[b], cH[:, b][:, None]) + loc_H[b])
    Ho = np.concatenate(outH, 1).astype(output_dtype)
    if not return_prefix:
        return Ho
    return np.concatenate(outP, 1).astype(output_dtype), Ho


# --------------------------------------------------------------------------
# Headed forms.  The reference never wraps these in a function of its own; the
# survey composes them from affine_scan_sequential with U = f*I and
# V = (1-f) k v^T, followed by the readout einsum o_t = S_t^T q_t.
# --------------------------------------------------------------------------

def _fold(x):
    return x.reshape((-1,) + x.shape[2:])


def gated_scan_dense(q, k, v, f, *, state_dtype=np.float64, S0=None):
    """Literal composition: affine_scan_sequential(f*I, (1-f) k v^T) + readout.

    q,k: [B,H,T,dk]  v: [B,H,T,dv]  f: [B,H,T].  Materialises the dense f*I
    transitions exactly as the reference's operator would receive them.
    """
    B, Hh, T, dk = q.shape
    dv = v.shape[-1]
    fq = _fold(f).astype(state_dtype)
    U = fq[..., None, None] * np.eye(dk, dtype=state_dtype)
    Vin = (1.0 - fq)[..., None, None] * (_fold(k).astype(state_dtype)[..., :, None]
                                         * _fold(v).astype(state_dtype)[..., None, :])
    if S0 is not None:
        # a leading step with U=0, V=S0 injects the initial state
        U = np.concatenate([np.zeros_like(U[:, :1]), U], 1)
        Vin = np.concatenate([_fold(S0).astype(state_dtype)[:, None], Vin], 1)
    S = affine_scan_sequential(U, Vin, state_dtype=state_dtype, output_dtype=state_dtype)
    if S0 is not None:
        S = S[:, 1:]
    o = np.einsum("ntkv,ntk->ntv", S, _fold(q).astype(state_dtype))
    return o.reshape(B, Hh, T, dv)


def gated_scan(q, k, v, f, *, state_dtype=np.float64, S0=None, return_final=False):
    """Same recurrence as :func:`gated_scan_dense`, stepping the scalar gate
    directly (f*S == (f I) @ S element-for-element).  Returns o [B,H,T,dv]
    and optionally the final state S_T [B,H,dk,dv]."""
    B, Hh, T, dk = q.shape
    dv = v.shape[-1]
    qf, kf, vf = (_fold(x).astype(state_dtype) for x in (q, k, v))
    ff = _fold(f).astype(state_dtype)
    N = B * Hh
    S = np.zeros((N, dk, dv), state_dtype) if S0 is None else _fold(S0).astype(state_dtype).copy()
    o = np.empty((N, T, dv), state_dtype)
    for t in range(T):
        ft = ff[:, t][:, None, None]
        S = ft * S + (1.0 - ft) * (kf[:, t, :, None] * vf[:, t, None, :])
        o[:, t] = np.matmul(qf[:, t, None, :], S)[:, 0]
    o = o.reshape(B, Hh, T, dv)
    if return_final:
        return o, S.reshape(B, Hh, dk, dv)
    return o


def gated_scan_backward(q, k, v, f, do, *, state_dtype=np.float64):
    """Gradients of sum(o * do) w.r.t. q, k, v, f.

    Restates the chain rule through the reference's affine backward
    (affine_scan.py:65-124) with U = f I, V = (1-f) k v^T and the readout
    o_t = S_t^T q_t:  grad_H_t = q_t do_t^T;  Sigma from the reverse scan;
    df_t = tr(Sigma_t S_{t-1}^T) - <Sigma_t, k_t v_t^T>,
    dk_t = (1-f_t) Sigma_t v_t,  dv_t = (1-f_t) Sigma_t^T k_t,  dq_t = S_t do_t.
    """
    B, Hh, T, dk = q.shape
    dv = v.shape[-1]
    qf, kf, vf, dof = (_fold(x).astype(state_dtype) for x in (q, k, v, do))
    ff = _fold(f).astype(state_dtype)
    N = B * Hh
    S_all = np.empty((N, T + 1, dk, dv), state_dtype)
    S_all[:, 0] = 0
    S = np.zeros((N, dk, dv), state_dtype)
    for t in range(T):
        ft = ff[:, t][:, None, None]
        S = ft * S + (1.0 - ft) * (kf[:, t, :, None] * vf[:, t, None, :])
        S_all[:, t + 1] = S
    dq = np.matmul(S_all[:, 1:], dof[..., None])[..., 0]
    dk_ = np.empty_like(kf)
    dv_ = np.empty_like(vf)
    df = np.empty_like(ff)
    carry = np.zeros((N, dk, dv), state_dtype)
    for t in range(T - 1, -1, -1):
        sig = qf[:, t, :, None] * dof[:, t, None, :] + carry
        w = (1.0 - ff[:, t])[:, None]
        sv = np.matmul(sig, vf[:, t, :, None])[..., 0]          # Sigma_t v_t
        dk_[:, t] = w * sv
        dv_[:, t] = w * np.matmul(kf[:, t, None, :], sig)[:, 0]  # Sigma_t^T k_t
        # <Sigma, S_{t-1}> - <Sigma, k v^T> = <Sigma, S_{t-1}> - k . (Sigma v)
        df[:, t] = (sig * S_all[:, t]).sum((1, 2)) - (kf[:, t] * sv).sum(1)
        carry = ff[:, t][:, None, None] * sig
    r = lambda x: x.reshape((B, Hh) + x.shape[1:])
    return r(dq), r(dk_), r(dv_), r(df)


def matrix_scan(A, q, k, v, f, *, state_dtype=np.float64):
    """Dense-transition headed scan:
    S_t = A_t S_{t-1} + (1-f_t) k_t v_t^T,  o_t = S_t^T q_t.
    A: [B,H,T,dk,dk]; composition of affine_scan_sequential with the readout."""
    B, Hh, T, dk = q.shape
    dv = v.shape[-1]
    ff = _fold(f).astype(state_dtype)
    U = _fold(A).astype(state_dtype)
    Vin = (1.0 - ff)[..., None, None] * (_fold(k).astype(state_dtype)[..., :, None]
                                         * _fold(v).astype(state_dtype)[..., None, :])
    S = affine_scan_sequential(U, Vin, state_dtype=state_dtype, output_dtype=state_dtype)
    o = np.einsum("ntkv,ntk->ntv", S, _fold(q).astype(state_dtype))
    return o.reshape(B, Hh, T, dv)


def matrix_scan_backward(A, q, k, v, f, do, *, state_dtype=np.float64):
    """Gradients of sum(o*do) for :func:`matrix_scan` via the reference's
    affine backward (affine_scan.py:65-124).  Returns dA, dq, dk, dv, df."""
    B, Hh, T, dk = q.shape
    dv = v.shape[-1]
    qf, kf, vf, dof = (_fold(x).astype(state_dtype) for x in (q, k, v, do))
    ff = _fold(f).astype(state_dtype)
    U = _fold(A).astype(state_dtype)
    kv = kf[..., :, None] * vf[..., None, :]
    Vin = (1.0 - ff)[..., None, None] * kv
    S = affine_scan_sequential(U, Vin, state_dtype=state_dtype, output_dtype=state_dtype)
    dq = np.einsum("ntkv,ntv->ntk", S, dof)
    gH = qf[..., :, None] * dof[..., None, :]
    gU, gV = affine_scan_sequential_backward(U, Vin, gH, state_dtype=state_dtype)
    w = (1.0 - ff)[..., None]
    dk_ = w * np.einsum("ntkv,ntv->ntk", gV, vf)
    dv_ = w * np.einsum("ntkv,ntk->ntv", gV, kf)
    df = -np.einsum("ntkv,ntkv->nt", gV, kv)
    r = lambda x: x.reshape((B, Hh) + x.shape[1:])
    return r(gU), r(dq), r(dk_), r(dv_), r(df)


# --------------------------------------------------------------------------
# Streaming forms of the dense-transition scan for full-size parity checks:
# the same recurrence as affine_scan_sequential (affine_scan.py:14-62) and its
# backward (affine_scan.py:65-124), stepped one t at a time so that no
# [N, T, d, d] state history is materialised (config 3 would need 4.3 GB of
# float64 states).  Inputs may be float32; every step runs in state_dtype.
# --------------------------------------------------------------------------

def matrix_scan_stream(A, q, k, v, f, *, state_dtype=np.float64, S0=None, return_final=False):
    """o_t = S_t^T q_t with S_t = A_t S_{t-1} + (1-f_t) k_t v_t^T
    (affine_scan.py:47-55's loop body with U = A, V = (1-f) k v^T).
    A: [B,H,T,dk,dk]; q, k: [B,H,T,dk]; v: [B,H,T,dv]; f: [B,H,T]."""
    B, Hh, T, dk = q.shape
    dv = v.shape[-1]
    Af, qf, kf, vf, ff = (_fold(x) for x in (A, q, k, v, f))
    N = B * Hh
    S = np.zeros((N, dk, dv), state_dtype) if S0 is None else _fold(S0).astype(state_dtype).copy()
    o = np.empty((N, T, dv), state_dtype)
    for t in range(T):
        w = (1.0 - ff[:, t].astype(state_dtype))[:, None, None]
        S = np.matmul(Af[:, t].astype(state_dtype), S) + w * (
            kf[:, t, :, None].astype(state_dtype) * vf[:, t, None, :].astype(state_dtype))
        o[:, t] = np.einsum("nkv,nk->nv", S, qf[:, t].astype(state_dtype))
    o = o.reshape(B, Hh, T, dv)
    if return_final:
        return o, S.reshape(B, Hh, dk, dv)
    return o


def matrix_scan_backward_stream(A, q, k, v, f, do, *, state_dtype=np.float64, S0=None,
                                chunk=64):
    """Gradients of sum(o * do) for :func:`matrix_scan_stream`, the chain rule
    through affine_scan.py:65-124 (Sigma_t = g_t + A_{t+1}^T Sigma_{t+1},
    dA_t = Sigma_t S_{t-1}^T) with g_t = q_t do_t^T and V = (1-f) k v^T.
    States are checkpointed every `chunk` steps and recomputed inside a chunk
    during the reverse sweep.  Returns dA (float32), dq, dk, dv, df and dS0."""
    B, Hh, T, dk = q.shape
    dv = v.shape[-1]
    Af, qf, kf, vf, ff, dof = (_fold(x) for x in (A, q, k, v, f, do))
    N = B * Hh
    sd = state_dtype
    S = np.zeros((N, dk, dv), sd) if S0 is None else _fold(S0).astype(sd).copy()
    nchk = (T + chunk - 1) // chunk
    ck = np.empty((nchk, N, dk, dv), sd)

    def step(S, t):
        w = (1.0 - ff[:, t].astype(sd))[:, None, None]
        return np.matmul(Af[:, t].astype(sd), S) + w * (
            kf[:, t, :, None].astype(sd) * vf[:, t, None, :].astype(sd))

    for t in range(T):
        if t % chunk == 0:
            ck[t // chunk] = S
        S = step(S, t)
    dA = np.empty(Af.shape, np.float32)
    dq = np.empty((N, T, dk), sd)
    dk_ = np.empty((N, T, dk), sd)
    dv_ = np.empty((N, T, dv), sd)
    df = np.empty((N, T), sd)
    carry = np.zeros((N, dk, dv), sd)    # A_{t+1}^T Sigma_{t+1}
    for c in range(nchk - 1, -1, -1):
        t0, t1 = c * chunk, min(T, (c + 1) * chunk)
        hist = np.empty((t1 - t0 + 1, N, dk, dv), sd)   # S_{t0-1} .. S_{t1-1}
        hist[0] = ck[c]
        for t in range(t0, t1):
            hist[t - t0 + 1] = step(hist[t - t0], t)
        for t in range(t1 - 1, t0 - 1, -1):
            St, Sp = hist[t - t0 + 1], hist[t - t0]
            qt, dot = qf[:, t].astype(sd), dof[:, t].astype(sd)
            kt, vt = kf[:, t].astype(sd), vf[:, t].astype(sd)
            dq[:, t] = np.einsum("nkv,nv->nk", St, dot)
            sig = qt[:, :, None] * dot[:, None, :] + carry
            dA[:, t] = np.matmul(sig, np.swapaxes(Sp, 1, 2))
            w = (1.0 - ff[:, t].astype(sd))[:, None]
            dk_[:, t] = w * np.einsum("nkv,nv->nk", sig, vt)
            dv_[:, t] = w * np.einsum("nkv,nk->nv", sig, kt)
            df[:, t] = -np.einsum("nkv,nk,nv->n", sig, kt, vt)
            carry = np.matmul(np.swapaxes(Af[:, t].astype(sd), 1, 2), sig)
    r = lambda x: x.reshape((B, Hh) + x.shape[1:])
    return r(dA), r(dq), r(dk_), r(dv_), r(df), r(carry)


# --------------------------------------------------------------------------
# Torch form of the reference's CPU path, for the timed CPU baseline: the
# same per-step batched matmul loop affine_scan.py:47-55 runs (fp32 state,
# dense f*I transitions, one bmm plus one add per step, the states stacked at
# the end), followed by the readout einsum.  Timing this form measures the
# reference's own CPU code path (torch ops on the host cores); the numpy
# restatement above is the checker.
# --------------------------------------------------------------------------

def gated_scan_torch_reference_path(q, k, v, f):
    """q, k, v: [B, H, T, d] float32 torch tensors, f: [B, H, T]; returns o."""
    import torch
    B, Hh, T, dk = q.shape
    dv = v.shape[-1]
    N = B * Hh
    ff = f.reshape(N, T).float()
    U = ff[..., None, None] * torch.eye(dk, dtype=torch.float32)
    Vin = (1.0 - ff)[..., None, None] * (k.reshape(N, T, dk, 1).float() * v.reshape(N, T, 1, dv).float())
    H = torch.zeros(N, dk, dv, dtype=torch.float32)
    states = []
    for t in range(T):
        H = torch.bmm(U[:, t], H) + Vin[:, t]
        states.append(H)
    S = torch.stack(states, dim=1)
    o = torch.einsum("ntkv,ntk->ntv", S, q.reshape(N, T, dk).float())
    return o.reshape(B, Hh, T, dv)
