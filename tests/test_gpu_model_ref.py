"""The MOGT model path on the GPU against the REFERENCE model's own outputs.

tests/golden/make_golden_model.py ran the reference MOGTModel
(model_mogt.py) on the CPU with its sequential scan and saved its weights,
final hidden states and training gradients.  Here the same weights are
loaded into mogt_b200's model, whose blocks call the B200 drop-in
(triton_affine_scan_hybrid, the scan the reference model imports for
scan_impl="triton_hybrid") and the connection-map kernel, with autograd on:
the forward and the gradients of the same loss must agree (fp32: 1e-4
relative on the hidden states, 1e-3 on the gradients)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GRADS = ["blocks.0.phi_conn.weight", "blocks.0.phi_value_gate.weight", "blocks.1.theta_read.weight",
         "embedding.weight"]


@pytest.mark.parametrize("connection", ["cayley", "matrix_exp"])
def test_reference_model_outputs_and_gradients(golden, connection):
    from mogt_b200.backbone import MOGTModel, configure_identity_coupled
    d = golden("model_small")
    m = MOGTModel(97, 64, 2, 16)
    configure_identity_coupled(m, damping=0.999)
    for blk in m.blocks:
        blk.connection_impl = connection
    state = {k.split("/state/", 1)[1]: torch.from_numpy(v) for k, v in d.items()
             if k.startswith(f"{connection}/state/")}
    m.load_state_dict(state, strict=True)
    m = m.cuda().train()
    ids = torch.from_numpy(d[f"{connection}/ids"]).cuda()
    hidden = m(ids)
    ref_h = d[f"{connection}/hidden"]
    err = np.abs(hidden.detach().cpu().numpy() - ref_h).max() / np.abs(ref_h).max()
    assert err <= 1e-4, err
    logits = hidden @ m.embedding.weight.t()
    loss = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, 97), ids[:, 1:].reshape(-1))
    assert abs(float(loss.detach()) - float(d[f"{connection}/loss"])) <= 1e-5 * float(d[f"{connection}/loss"])
    named = dict(m.named_parameters())
    grads = torch.autograd.grad(loss, [named[n] for n in GRADS])
    for n, g in zip(GRADS, grads):
        ref = d[f"{connection}/grad/{n}"]
        e = np.abs(g.cpu().numpy() - ref).max() / np.abs(ref).max()
        assert e <= 1e-3, (n, e)
