"""Golden vectors for the chunked linear cross-entropy, made by running the
REFERENCE's own ``chunked_lm_loss.chunked_linear_cross_entropy`` (lkcfqy/MOGT
chunked_lm_loss.py) on the CPU in the build container.

Usage (build container only; the reference tree is not on GPU boxes):
    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden_ce.py <reference_dir>

Case: B=2, L=75, D=48, V=517, chunk_size=64 (a ragged last chunk), seed 0,
hidden ~ N(0,1), weight ~ 0.05 N(0,1), labels uniform with every 9th token
set to -100 (F.cross_entropy's ignored label); upstream gradient 1.7.
"""
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main():
    sys.dont_write_bytecode = True
    sys.path.insert(0, sys.argv[1])
    import chunked_lm_loss as ref  # the reference module, read-only
    g = torch.Generator().manual_seed(0)
    B, L, D, V = 2, 75, 48, 517
    h = torch.randn(B, L, D, generator=g, dtype=torch.float32).requires_grad_(True)
    w = (0.05 * torch.randn(V, D, generator=g, dtype=torch.float32)).requires_grad_(True)
    labels = torch.randint(0, V, (B, L), generator=g)
    labels.view(-1)[::9] = -100
    loss = ref.chunked_linear_cross_entropy(h, w, labels, chunk_size=64)
    dh, dw = torch.autograd.grad(loss, (h, w), grad_outputs=torch.tensor(1.7))
    np.savez_compressed(HERE / "chunked_ce.npz", hidden=h.detach().numpy(), weight=w.detach().numpy(),
                        labels=labels.numpy(), loss=loss.detach().numpy(), grad_out=np.float32(1.7),
                        d_hidden=dh.numpy(), d_weight=dw.numpy())


if __name__ == "__main__":
    main()
