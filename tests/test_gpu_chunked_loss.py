"""Chunked linear cross-entropy on the GPU against the reference's own
function (golden vectors from tests/golden/make_golden_ce.py) and, at a
larger size, against torch's F.cross_entropy in float64.  fp32 arithmetic:
1e-5 relative on the loss, 1e-4 on the gradients."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_matches_reference_golden(golden):
    from mogt_b200.chunked_lm_loss import chunked_linear_cross_entropy
    d = golden("chunked_ce")
    h = torch.from_numpy(d["hidden"]).cuda().requires_grad_(True)
    w = torch.from_numpy(d["weight"]).cuda().requires_grad_(True)
    lab = torch.from_numpy(d["labels"]).cuda()
    loss = chunked_linear_cross_entropy(h, w, lab, chunk_size=64)
    assert abs(float(loss.detach()) - float(d["loss"])) <= 1e-5 * abs(float(d["loss"]))
    dh, dw = torch.autograd.grad(loss, (h, w), grad_outputs=torch.tensor(float(d["grad_out"]), device="cuda"))
    for got, ref in ((dh, d["d_hidden"]), (dw, d["d_weight"])):
        assert np.abs(got.cpu().numpy() - ref).max() <= 1e-4 * np.abs(ref).max()


def test_lm_head_size_against_torch():
    from mogt_b200.chunked_lm_loss import chunked_linear_cross_entropy
    g = torch.Generator(device="cuda").manual_seed(1)
    B, L, D, V = 2, 1000, 256, 32000
    h = torch.randn(B, L, D, generator=g, device="cuda")
    w = 0.02 * torch.randn(V, D, generator=g, device="cuda")
    lab = torch.randint(0, V, (B, L), generator=g, device="cuda")
    loss = chunked_linear_cross_entropy(h, w, lab, chunk_size=512)
    ref = torch.nn.functional.cross_entropy(h.double().reshape(-1, D) @ w.double().t(), lab.reshape(-1))
    assert abs(float(loss) - float(ref)) <= 1e-5 * abs(float(ref))


def test_errors():
    from mogt_b200.chunked_lm_loss import chunked_linear_cross_entropy
    h = torch.zeros(1, 4, 8, device="cuda")
    w = torch.zeros(10, 8, device="cuda")
    with pytest.raises(ValueError):
        chunked_linear_cross_entropy(h, w, torch.zeros(1, 4, dtype=torch.int64, device="cuda"), chunk_size=0)
    with pytest.raises(ValueError):
        chunked_linear_cross_entropy(h, w, torch.full((1, 4), 10, device="cuda"), chunk_size=2)
    with pytest.raises(ValueError):
        chunked_linear_cross_entropy(h[0], w, torch.zeros(1, 4, dtype=torch.int64, device="cuda"), chunk_size=2)
