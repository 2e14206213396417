"""Memory-efficient linear cross-entropy for tied LM heads, on the GPU.

Drop-in for the reference module of the same name (chunked_lm_loss.py:5-80):
same function, arguments, errors and result.  Per chunk of tokens the fp32
logits are one cuBLAS GEMM (as in the reference); the softmax cross-entropy
that follows is one kernel pass over the chunk (mogt_ce_rows_fwd: online
max / sum-of-exp per row, writing each row's log-sum-exp and loss), and the
backward recomputes the chunk's logits and turns them into the softmax
gradient in place with one more pass (mogt_ce_rows_bwd, using the saved
log-sum-exp) before the two GEMMs of the weight and hidden-state gradients.
Labels of -100 contribute no loss (F.cross_entropy's default ignore_index)
and, like the reference's probs[arange, labels] -= 1, subtract the one-hot
at column V - 100 in the backward.
"""
from __future__ import annotations

import torch

from . import _native as N

__all__ = ["chunked_linear_cross_entropy", "_ChunkedLinearCrossEntropy"]


def _check_labels(labels, V):
    bad = (labels >= V) | ((labels < 0) & (labels != -100))
    if bool(bad.any()):
        raise ValueError("labels must lie in [0, V) or equal -100")


class _ChunkedLinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden_states, weight, labels, chunk_size: int):
        if hidden_states.ndim != 3:
            raise ValueError("hidden_states must be [B, L, D]")
        if labels.shape != hidden_states.shape[:2]:
            raise ValueError("labels must be [B, L]")
        if weight.ndim != 2 or weight.shape[1] != hidden_states.shape[-1]:
            raise ValueError("weight must be [V, D]")
        chunk_size = int(chunk_size)
        if chunk_size <= 0:
            raise ValueError("chunk_size must be positive")
        if hidden_states.device.type != "cuda":
            raise ValueError("chunked_linear_cross_entropy requires CUDA tensors")
        B, L, D = hidden_states.shape
        V = weight.shape[0]
        total = B * L
        hidden = hidden_states.reshape(total, D)
        lab = labels.reshape(total).to(torch.int64).contiguous()
        _check_labels(lab, V)
        wf = weight.float()
        lse = torch.empty(total, dtype=torch.float32, device=hidden.device)
        loss_rows = torch.empty(total, dtype=torch.float32, device=hidden.device)
        lib = N.lib()
        stream = N.stream_ptr(hidden.device)
        with torch.no_grad(), torch.cuda.device(hidden.device):
            for s in range(0, total, chunk_size):
                e = min(s + chunk_size, total)
                logits = hidden[s:e].float().matmul(wf.t()).contiguous()
                st = lib.mogt_ce_rows_fwd(N.ptr(logits), N.ptr(lab[s:e]), e - s, V, N.ptr(lse[s:e]),
                                          N.ptr(loss_rows[s:e]), stream)
                N.check(st, "mogt_ce_rows_fwd")
        ctx.save_for_backward(hidden_states, weight, lab, lse)
        ctx.chunk_size = chunk_size
        return loss_rows.sum() / total

    @staticmethod
    def backward(ctx, grad_output):
        hidden_states, weight, lab, lse = ctx.saved_tensors
        B, L, D = hidden_states.shape
        V = weight.shape[0]
        total = B * L
        hidden = hidden_states.reshape(total, D)
        grad_hidden = torch.empty_like(hidden)
        grad_weight = torch.zeros_like(weight, dtype=torch.float32)
        wf = weight.float()
        scale = float(grad_output.float().item()) / float(total)
        lib = N.lib()
        stream = N.stream_ptr(hidden.device)
        with torch.cuda.device(hidden.device):
            for s in range(0, total, ctx.chunk_size):
                e = min(s + ctx.chunk_size, total)
                hc = hidden[s:e].float()
                probs = hc.matmul(wf.t()).contiguous()
                st = lib.mogt_ce_rows_bwd(N.ptr(probs), N.ptr(lab[s:e]), N.ptr(lse[s:e]), e - s, V,
                                          scale, stream)
                N.check(st, "mogt_ce_rows_bwd")
                grad_hidden[s:e] = probs.matmul(wf).to(hidden_states.dtype)
                grad_weight.addmm_(probs.t(), hc)
        return grad_hidden.view_as(hidden_states), grad_weight.to(weight.dtype), None, None


def chunked_linear_cross_entropy(hidden_states, weight, labels, *, chunk_size: int):
    """Mean cross-entropy of softmax(hidden_states @ weight^T) against labels,
    computed chunk_size tokens at a time; only hidden states, labels, the
    weight and one float per token are kept for the backward."""
    return _ChunkedLinearCrossEntropy.apply(hidden_states, weight, labels, int(chunk_size))
