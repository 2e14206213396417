"""Device-side failures reach the caller.  No test makes a kernel time out:
the timeout record a kernel would leave (MOGT_ERR_TIMEOUT in the workspace
header's sticky error word) is written into the header from the host, and
the tests check that the library reports it and then recovers."""
import pytest
import torch

from tests.helpers import headed_bf16

pytestmark = pytest.mark.gpu


def _entry(dev, family):
    from mogt_b200 import _native as N
    key = [k for k in N.workspaces._ws if k[0] == dev.index and k[2] == family]
    assert key, family
    return N.workspaces._ws[key[0]]


def _plant_timeout(w, unit=7):
    w.buf[12:20].view(torch.int32).copy_(torch.tensor([5, unit], dtype=torch.int32))


def test_check_errors_raises_then_clears():
    import mogt_b200
    from mogt_b200 import _native as N
    dev = torch.device("cuda", 0)
    q, k, v, f = (t.to(dev) for t in headed_bf16(1, 2, 700, seed=1))
    mogt_b200.gated_scan(q, k, v, f)
    N.check_errors(dev)                      # nothing recorded
    _plant_timeout(_entry(dev, "gated_fwd"))
    with pytest.raises(N.DeviceTimeout, match="unit 7"):
        N.check_errors(dev)
    N.check_errors(dev)                      # the read cleared the record
    assert all(e == 0 for e in N.workspace_errors(dev))


def test_next_call_raises_deferred():
    import mogt_b200
    from mogt_b200 import _native as N
    dev = torch.device("cuda", 0)
    q, k, v, f = (t.to(dev) for t in headed_bf16(1, 2, 700, seed=2))
    o_ref = mogt_b200.gated_scan(q, k, v, f)
    w = _entry(dev, "gated_fwd")
    _plant_timeout(w, unit=3)
    mogt_b200.gated_scan(q, k, v, f)         # its status copy sees the record
    torch.cuda.synchronize()
    with pytest.raises(N.DeviceTimeout, match="unit 3"):
        mogt_b200.gated_scan(q, k, v, f)
    o = mogt_b200.gated_scan(q, k, v, f)     # recovered
    assert torch.equal(o, o_ref)
