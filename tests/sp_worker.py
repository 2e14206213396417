"""torchrun worker for tests/test_gpu_sp.py: each rank scans its contiguous
segment of one sequence with the NCCL carry exchange; rank 0 checks the
concatenated result against a one-GPU scan of the whole sequence."""
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main():
    T = int(sys.argv[1])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    from mogt_b200 import ops
    from mogt_b200.sp import gated_scan_sp
    from tests.helpers import headed_bf16
    q, k, v, f = (t.to(dev) for t in headed_bf16(1, 12, T, seed=7))
    seg = T // world
    sl = slice(rank * seg, (rank + 1) * seg)
    o = gated_scan_sp(q[:, :, sl].contiguous(), k[:, :, sl].contiguous(), v[:, :, sl].contiguous(),
                      f[:, :, sl].contiguous(), output_dtype=torch.float32)
    outs = [torch.empty_like(o) for _ in range(world)]
    dist.all_gather(outs, o)
    ok = 1
    if rank == 0:
        full = torch.cat(outs, 2)
        ref, _, _, _ = ops.gated_scan_fwd(q, k, v, f, output_dtype=torch.float32)
        err = float((full - ref).abs().max() / ref.abs().max())
        print(f"sp world={world} T={T} rel_err={err:.3e}", flush=True)
        ok = int(err <= 2e-3 and torch.isfinite(full).all().item())
    flag = torch.tensor([ok], device=dev)
    dist.broadcast(flag, 0)
    dist.destroy_process_group()
    sys.exit(0 if flag.item() else 1)


if __name__ == "__main__":
    main()
