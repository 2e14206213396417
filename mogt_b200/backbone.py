"""MOGT backbone (embedding -> N x MOGT block -> final RMSNorm) whose affine
scan runs on libmogt_scan.so.

This is the caller of the scan in the reference (model_mogt.py:32-287,
MOGTBlock / MOGTModel), re-implemented so the backbone benchmark (BASELINE
config 4) runs where the reference tree is not available.  Module and
parameter names follow the reference, so a reference state_dict loads
unchanged (`load_state_dict`), and the block's options keep the reference's
attribute names and defaults (model_mogt.py:71-122, 141-183, 243-256):
connection_impl ("matrix_exp" | "cayley" | "identity"), connection_damping,
phi_value_gate (attached by the caller, scalar or rank-wise),
value_gate_input_mode ("current" | "current_prev" | "current_prev_prefix"),
couple_forget_to_value_gate.  The transport gate and the residual gating
options of the research code are not carried over.

The scan is `scan_fn(U, V, output_dtype)`; the default is
mogt_b200.triton_scan.triton_affine_scan_hybrid, the drop-in of the
reference's own `scan_impl = "triton_hybrid"` path.  Another function can be
passed (tests use it to compare against the reference's sequential scan).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops, triton_scan

__all__ = ["RMSNorm", "SwiGLU", "MOGTBlock", "MOGTModel", "configure_identity_coupled"]


def _b200_scan(U, V, output_dtype):
    return triton_scan.triton_affine_scan_hybrid(U, V, output_dtype=output_dtype)


class RMSNorm(nn.Module):
    """x / rms(x) in fp32, cast back, times a learned gain."""

    def __init__(self, d_model: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d_model))

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return y.type_as(x) * self.weight


class SwiGLU(nn.Module):
    def __init__(self, d_model: int, hidden: int):
        super().__init__()
        self.w1 = nn.Linear(d_model, hidden, bias=False)
        self.w2 = nn.Linear(d_model, hidden, bias=False)
        self.w3 = nn.Linear(hidden, d_model, bias=False)

    def forward(self, x):
        return self.w3(F.silu(self.w1(x)) * self.w2(x))


class MOGTBlock(nn.Module):
    """Transport U_t (R x R) and value V_t (R x C) from the normalised input,
    the affine scan H_t = U_t H_{t-1} + V_t, readout theta_read(RMSNorm(H)),
    residual, then a SwiGLU feed-forward with its own residual."""

    def __init__(self, d_model: int, r: int = 16, scan_fn=None):
        super().__init__()
        if d_model % r:
            raise ValueError("d_model must be divisible by r")
        self.d_model, self.r, self.c = d_model, r, d_model // r
        self.connection_impl = "matrix_exp"
        self.connection_damping = 0.999
        self.register_buffer("_identity_r", torch.eye(r), persistent=False)
        self.norm_mogt = RMSNorm(d_model)
        self.phi_conn = nn.Linear(d_model, r * r, bias=False)
        self.phi_val = nn.Linear(d_model, r * self.c, bias=False)
        self.norm_out = RMSNorm(d_model)
        self.theta_read = nn.Linear(r * self.c, d_model, bias=False)
        self.norm_ffn = RMSNorm(d_model)
        hidden = 256 * math.ceil(int(8 * d_model / 3) / 256)
        self.ffn = SwiGLU(d_model, hidden)
        self.scan_fn = scan_fn or _b200_scan

    def transport(self, x_norm):
        B, L, _ = x_norm.shape
        impl = getattr(self, "connection_impl", "matrix_exp")
        damping = float(getattr(self, "connection_damping", 0.999))
        if impl == "identity":
            U = self._identity_r.view(1, 1, self.r, self.r).expand(B, L, self.r, self.r)
        elif x_norm.is_cuda:
            # on the GPU: the connection-map kernel (mogt_connection_map)
            from .connection import connection_map
            return connection_map(self.phi_conn(x_norm).view(B, L, self.r, self.r), impl, damping,
                                  output_dtype=x_norm.dtype)
        else:
            # CPU tensors (the parity harness against the reference model)
            A = self.phi_conn(x_norm).view(B, L, self.r, self.r)
            A = ((A - A.transpose(-2, -1)) / self.r).float()
            if impl == "matrix_exp":
                U = torch.matrix_exp(A)
            elif impl == "cayley":
                eye = self._identity_r.view(1, 1, self.r, self.r)
                U = torch.linalg.solve(eye - 0.5 * A, eye + 0.5 * A)
            else:
                raise ValueError(f"unsupported connection_impl: {impl}")
        return (U * damping).to(x_norm.dtype)

    def value_gate_input(self, x_norm, prefix):
        mode = getattr(self, "value_gate_input_mode", "current")
        parts = [x_norm]
        if "prev" in mode:
            parts.append(F.pad(x_norm, (0, 0, 1, 0))[:, :-1])
        if "prefix" in mode:
            p = (torch.zeros_like(x_norm[:, :1]) if prefix is None
                 else prefix.to(x_norm.dtype).view(x_norm.size(0), 1, -1))
            parts.append(p.expand_as(x_norm))
        return parts[0] if len(parts) == 1 else torch.cat(parts, -1)

    def _fused_identity_path(self, x, gate_lin):
        """The identity connection with the forget gate coupled to the value
        gate makes U_t diagonal: the scan and norm_out then run as one fused
        kernel (mogt_diag_scan_norm_fwd) without materialising U or the fp32
        states; with autograd on, its reverse-time chunked backward
        (mogt_diag_scan_norm_bwd) gives the gradients.  Used with the default
        B200 scan."""
        return (getattr(self, "fused_identity_scan", True)
                and getattr(self, "connection_impl", "matrix_exp") == "identity"
                and gate_lin is not None
                and getattr(self, "couple_forget_to_value_gate", False)
                and self.scan_fn is _b200_scan
                and x.is_cuda
                and self.c % 2 == 0 and (self.r * self.c) % 64 == 0 and self.r * self.c <= 1024)

    def _gate_logits(self, x_norm, prefix, gate_lin):
        """phi_value_gate(value_gate_input(x_norm, prefix)) without building
        the concatenated [x_t, x_{t-1}, x_prefix] input: one GEMM of x_norm
        against the current and previous-token weight blocks (fp32
        accumulation), the previous-token part shifted by one step, the prefix
        part once per sequence, the bias, then one rounding to the dtype the
        concatenated linear would output (bf16 under bf16 autocast).  Equal to
        the concatenated form up to fp32 summation order."""
        mode = getattr(self, "value_gate_input_mode", "current")
        B, L, D = x_norm.shape
        prev, pre = "prev" in mode, "prefix" in mode
        W = gate_lin.weight
        if W.size(1) != (1 + prev + pre) * D:
            return gate_lin(self.value_gate_input(x_norm, prefix)).float()
        bf = torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
        dt = torch.bfloat16 if bf else x_norm.dtype

        def mm(a, w):
            a, w = a.to(dt), w.to(dt)
            with torch.autocast("cuda", enabled=False):
                return torch.mm(a, w.t(), out_dtype=torch.float32) if bf else torch.mm(a, w.t()).float()

        n = W.size(0)
        wx = torch.cat([W[:, :D], W[:, D:2 * D]], 0) if prev else W[:, :D]
        y = mm(x_norm.reshape(B * L, D), wx).view(B, L, -1)
        logit = y[..., :n].clone()
        if prev and L > 1:
            logit[:, 1:] += y[:, :-1, n:]
        if pre:
            p = (torch.zeros(B, D, device=x_norm.device, dtype=x_norm.dtype) if prefix is None
                 else prefix.to(x_norm.dtype).reshape(B, D))
            logit += mm(p, W[:, (1 + prev) * D:])[:, None]
        if gate_lin.bias is not None:
            logit += gate_lin.bias.float()
        return logit.to(dt).float() if bf else logit

    def forward(self, x, prefix_condition=None):
        B, L, D = x.shape
        x_norm = self.norm_mogt(x)
        gate_lin = getattr(self, "phi_value_gate", None)
        if self._fused_identity_path(x, gate_lin):
            with torch.autograd.profiler.record_function("mogt.value_projection"):
                V = self.phi_val(x_norm).view(B, L, self.r, self.c)
                if torch.is_grad_enabled():
                    # the concatenated-input linear, differentiable as is
                    z = gate_lin(self.value_gate_input(x_norm, prefix_condition)).float()
                else:
                    z = self._gate_logits(x_norm, prefix_condition, gate_lin)
                if z.size(-1) not in (1, self.r):
                    raise ValueError("phi_value_gate must output 1 or r gates")
                z = torch.sigmoid(z)
            with torch.autograd.profiler.record_function("mogt.fused_scan_norm"):
                # the readout GEMM consumes bf16 under bf16 autocast: write that directly
                y_dtype = (torch.bfloat16 if torch.is_autocast_enabled("cuda")
                           and torch.get_autocast_dtype("cuda") == torch.bfloat16 else torch.float32)
                damping = float(getattr(self, "connection_damping", 0.999))
                if torch.is_grad_enabled():
                    y = ops.DiagScanNormFn.apply(V, z, self.norm_out.weight, None, damping,
                                                 self.norm_out.eps, y_dtype)
                else:
                    y, _ = ops.diag_scan_norm(V, z, self.norm_out.weight, damping=damping,
                                              eps=self.norm_out.eps, output_dtype=y_dtype)
            with torch.autograd.profiler.record_function("mogt.readout"):
                x = x + self.theta_read(y.view(B, L, D))
            with torch.autograd.profiler.record_function("mogt.ffn"):
                x = x + self.ffn(self.norm_ffn(x))
            return x
        with torch.autograd.profiler.record_function("mogt.connection_map"):
            U = self.transport(x_norm)
        with torch.autograd.profiler.record_function("mogt.value_projection"):
            V = self.phi_val(x_norm).view(B, L, self.r, self.c)
            if gate_lin is not None:
                z = gate_lin(self.value_gate_input(x_norm, prefix_condition)).float()
                if z.size(-1) not in (1, self.r):
                    raise ValueError("phi_value_gate must output 1 or r gates")
                z = torch.sigmoid(z).view(B, L, z.size(-1), 1)
                V = V * z.to(V.dtype)
                if getattr(self, "couple_forget_to_value_gate", False):
                    U = U * (1.0 - z).to(U.dtype)
        with torch.autograd.profiler.record_function("mogt.affine_scan"):
            H = self.scan_fn(U, V, U.dtype)
        with torch.autograd.profiler.record_function("mogt.readout"):
            x = x + self.theta_read(self.norm_out(H.reshape(B, L, D)))
        with torch.autograd.profiler.record_function("mogt.ffn"):
            x = x + self.ffn(self.norm_ffn(x))
        return x


class MOGTModel(nn.Module):
    def __init__(self, vocab_size: int, d_model: int = 768, num_layers: int = 12, r: int = 16,
                 scan_fn=None):
        super().__init__()
        self.embedding = nn.Embedding(vocab_size, d_model)
        self.blocks = nn.ModuleList([MOGTBlock(d_model, r, scan_fn) for _ in range(num_layers)])
        self.norm_f = RMSNorm(d_model)

    def forward(self, input_ids):
        x = self.embedding(input_ids)
        pos = getattr(self, "prefix_condition_position", None)
        prefix = None
        if pos is not None and -x.size(1) <= int(pos) < x.size(1):
            prefix = x[:, int(pos), :]
        for blk in self.blocks:
            x = blk(x, prefix_condition=prefix)
        return self.norm_f(x)


def configure_identity_coupled(model: MOGTModel, *, gate_bias: float = -2.0, rank_gate: bool = True,
                               input_mode: str = "current_prev_prefix", prefix_position: int = 1,
                               damping: float = 1.0):
    """The backbone-throughput configuration (benchmark_backbone_throughput.py:
    33-59 defaults): identity connection, damping 1.0, rank-wise value gate on
    [x_t, x_{t-1}, x_prefix] with zero weights and bias -2, forget coupled to
    the value gate, prefix condition at position 1."""
    mult = {"current": 1, "current_prev": 2, "current_prev_prefix": 3}[input_mode]
    for blk in model.blocks:
        blk.connection_impl = "identity"
        blk.connection_damping = damping
        ref = next(blk.parameters())
        lin = nn.Linear(mult * blk.d_model, blk.r if rank_gate else 1, bias=True).to(ref.device)
        nn.init.zeros_(lin.weight)
        nn.init.constant_(lin.bias, gate_bias)
        blk.phi_value_gate = lin
        blk.value_gate_input_mode = input_mode
        blk.couple_forget_to_value_gate = True
    model.prefix_condition_position = prefix_position
    return model
