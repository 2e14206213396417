"""Sequence-parallel gated scan.

One long sequence is split into contiguous segments, one per rank (rank r
holds steps [r*T_loc, (r+1)*T_loc)).  The scan's carry is associative:
a segment maps an incoming state X to  A_r X + S_r  (A_r = product of its
gates, S_r = its state from a zero start), the same algebra as the block
carries of the reference (affine_scan.py:250-271).  So:

  1. every rank computes its segment carry (A_r, S_r) -- a state-only scan
     (no q, no output);
  2. the carries are all-gathered (NCCL over NVLink; one
     [world, B, H, 1 + dk*dv] fp32 tensor, ~197 KB per rank at H=12, 64x64);
  3. rank r combines the carries of ranks < r into its incoming state
     X_r = A_{r-1} X_{r-1} + S_{r-1} (X_0 = initial state or 0);
  4. every rank runs the output pass on its segment from X_r: this is the
     local correction pass that makes its outputs equal to a one-GPU scan.
     On the CUDA path it resumes the forward of step 1 (the chunk-local states
     are still in the workspace), so only the segment carry and the output
     kernel run again.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops

__all__ = ["gated_scan_sp", "combine_carries"]


def combine_carries(gathered: torch.Tensor, rank: int, dk: int, dv: int,
                    initial_state: torch.Tensor | None = None) -> torch.Tensor:
    """Incoming state of `rank` from the gathered carries.

    gathered: [world, B, H, 1 + dk*dv] with the decay A_r in [..., 0] and the
    zero-start final state S_r (row-major dk x dv) in [..., 1:].
    Returns X_rank: [B, H, dk, dv] in the carries' dtype (fp32 from the CUDA scan)."""
    world, B, H, _ = gathered.shape
    X = (torch.zeros(B, H, dk, dv, dtype=gathered.dtype, device=gathered.device)
         if initial_state is None else initial_state.to(gathered.dtype).clone())
    for r in range(rank):
        A = gathered[r, :, :, 0].view(B, H, 1, 1)
        S = gathered[r, :, :, 1:].view(B, H, dk, dv)
        X = A * X + S
    return X


def gated_scan_sp(q, k, v, f, *, group=None, output_dtype=None, initial_state=None,
                  local_fwd=None):
    """o for this rank's segment of a sequence split across the ranks of
    `group` (contiguous segments in rank order).  q, k: [B, H, T_loc, dk];
    v: [B, H, T_loc, dv]; f: [B, H, T_loc].  `initial_state` (rank 0's
    incoming state) must be given on every rank or on none.

    `local_fwd` defaults to the CUDA scan (mogt_b200.ops.gated_scan_fwd); it
    is a parameter only so the collective logic can be exercised by CPU
    tests with another local scan."""
    fwd = local_fwd or ops.gated_scan_fwd
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, H, _, dk = k.shape
    dv = v.shape[-1]
    with torch.autograd.profiler.record_function("mogt.sp.segment_carry"):
        _, S_loc, A_loc, _ = fwd(None, k, v, f, want_final=True, want_output=False)
    carry = torch.cat([A_loc.reshape(B, H, 1), S_loc.reshape(B, H, dk * dv)], -1).contiguous()
    # concatenated along dim 0 (the layout every backend accepts), then viewed
    flat = torch.empty((world * B,) + tuple(carry.shape[1:]), dtype=carry.dtype, device=carry.device)
    with torch.autograd.profiler.record_function("mogt.sp.all_gather"):
        dist.all_gather_into_tensor(flat, carry, group=group)
    gathered = flat.view((world,) + tuple(carry.shape))
    X = combine_carries(gathered, rank, dk, dv, initial_state)
    with torch.autograd.profiler.record_function("mogt.sp.local_scan"):
        if local_fwd is None and k.dtype == torch.bfloat16:
            o, _, _, _ = fwd(q, k, v, f, initial_state=X, output_dtype=output_dtype, resume=True)
        else:
            o, _, _, _ = fwd(q, k, v, f, initial_state=X, output_dtype=output_dtype)
    return o
