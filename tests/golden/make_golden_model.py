"""Golden vectors for the MOGT model path: the REFERENCE's own MOGTModel
(lkcfqy/MOGT model_mogt.py) run on the CPU in the build container with its
sequential scan (affine_scan.py:14-62), saved with its weights so the GPU
tests can load the same weights into mogt_b200's model and compare the
logits and the training gradients through the B200 scan.

Usage (build container only):
    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden_model.py <reference_dir>

Model: vocab 97, d_model 64, 2 layers, r 16, weights N(0, 0.02), the
benchmark's block configuration (rank-wise value gate on [x_t, x_{t-1},
x_prefix] coupled to the forget gate, prefix condition at position 1),
connection "cayley" and "matrix_exp" (damping 0.999), fp32, ids [2, 40]
seed 0; the model's final hidden states are saved, and the loss is the mean
cross-entropy of the tied-head logits (hidden @ embedding^T) against the ids
shifted by one.
"""
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
GRADS = ["blocks.0.phi_conn.weight", "blocks.0.phi_value_gate.weight", "blocks.1.theta_read.weight",
         "embedding.weight"]


def configure(model, d, connection):
    for blk in model.blocks:
        blk.scan_impl = "sequential"
        blk.connection_impl = connection
        blk.connection_damping = 0.999
        blk.phi_value_gate = torch.nn.Linear(3 * d, blk.r, bias=True)
        torch.nn.init.normal_(blk.phi_value_gate.weight, std=0.02)
        torch.nn.init.constant_(blk.phi_value_gate.bias, -2.0)
        blk.value_gate_input_mode = "current_prev_prefix"
        blk.couple_forget_to_value_gate = True
    model.prefix_condition_position = 1


def main():
    sys.dont_write_bytecode = True
    sys.path.insert(0, sys.argv[1])
    import model_mogt  # the reference module, read-only
    d, r, layers, vocab = 64, 16, 2, 97
    out = {}
    for connection in ("cayley", "matrix_exp"):
        torch.manual_seed(0)
        m = model_mogt.MOGTModel(vocab, d, layers, r)
        for p in m.parameters():
            torch.nn.init.normal_(p, std=0.02)
        configure(m, d, connection)
        ids = torch.randint(0, vocab, (2, 40))
        hidden = m(ids)
        logits = hidden @ m.embedding.weight.t()  # tied LM head
        loss = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, vocab), ids[:, 1:].reshape(-1))
        named = dict(m.named_parameters())
        grads = torch.autograd.grad(loss, [named[n] for n in GRADS])
        for k, v in m.state_dict().items():
            out[f"{connection}/state/{k}"] = v.detach().numpy()
        out[f"{connection}/ids"] = ids.numpy()
        out[f"{connection}/hidden"] = hidden.detach().numpy()
        out[f"{connection}/loss"] = loss.detach().numpy()
        for n, g in zip(GRADS, grads):
            out[f"{connection}/grad/{n}"] = g.numpy()
    np.savez_compressed(HERE / "model_small.npz", **out)


if __name__ == "__main__":
    main()
