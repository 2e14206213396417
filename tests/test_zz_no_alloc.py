"""The allocation-free gated-scan entry point (mogt_gated_scan_fwd_noalloc).

Some callers cannot allocate device memory -- a host runtime that owns all of
its GPU memory through its own allocator or budget, a foreign-language
binding with no way to reach that allocator, or code that must avoid the
implicit synchronisation of cudaMalloc.  For them the library keeps a fixed
16 MiB scratch array per GPU.  This test calls that entry point through the
C ABI, twice in a row (the second call reuses the array the first one left
behind), and checks both results against the regular entry point, which is
given a freshly allocated workspace.  It lives in its own file, collected
last, so a failure here never hides the other tests.
"""
import ctypes

import pytest
import torch

from tests.helpers import headed_bf16

pytestmark = pytest.mark.gpu
TOL_BF16 = 2e-2  # the bf16-input tolerance used by the other gated-scan tests


def _call(fn_name, q, k, v, f, o, S_fin, extra):
    from mogt_b200 import _native as N
    L = N.lib()
    B, H, T, d = q.shape
    args = [N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(f), N.ptr(o), None, N.ptr(S_fin), None, None,
            B * H, T, d, d, N.BF16, N.BF16]
    return getattr(L, fn_name)(*args, *extra, N.stream_ptr(q.device))


def test_noalloc_matches_workspace_entry_point_twice():
    from mogt_b200 import _native as N
    L = N.lib()
    dev = torch.device("cuda", 0)
    outs = []
    for seed, T in [(21, 5000), (22, 32768)]:
        q, k, v, f = (t.to(dev) for t in headed_bf16(1, 12, T, seed=seed))
        B, H = 1, 12
        # regular entry point with a caller-allocated, zeroed workspace
        nbytes = L.mogt_gated_scan_fwd_workspace_bytes(B * H, T, 64, 64, N.BF16)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        o_ref = torch.empty_like(q)
        S_ref = torch.empty(B, H, 64, 64, device=dev)
        assert _call("mogt_gated_scan_fwd", q, k, v, f, o_ref, S_ref,
                     [N.ptr(ws), ctypes.c_size_t(nbytes)]) == 0
        # the allocation-free entry point, called twice in a row
        for _ in range(2):
            o = torch.full_like(q, float("nan"))
            S = torch.full_like(S_ref, float("nan"))
            assert _call("mogt_gated_scan_fwd_noalloc", q, k, v, f, o, S, []) == 0
            torch.cuda.synchronize()
            err = (o.float() - o_ref.float()).abs().max() / o_ref.float().abs().max()
            assert float(err) <= TOL_BF16
            errS = (S - S_ref).abs().max() / S_ref.abs().max()
            assert float(errS) <= TOL_BF16
            outs.append(o)
            # no device-side wait gave up: the status reader says so
            err, unit = ctypes.c_int(-1), ctypes.c_uint32(0)
            assert L.mogt_gated_scan_fwd_noalloc_status(N.stream_ptr(dev), ctypes.byref(err),
                                                        ctypes.byref(unit)) == 0
            assert err.value == 0
    assert torch.isfinite(outs[-1].float()).all()


def test_noalloc_rejects_oversized_problems():
    from mogt_b200 import _native as N
    dev = torch.device("cuda", 0)
    q = torch.zeros(1, 1, 64, dtype=torch.bfloat16, device=dev)
    f = torch.ones(1, 64, device=dev)
    L = N.lib()
    # 4096 heads x 2^20 steps needs far more than the fixed 16 MiB of scratch
    st = L.mogt_gated_scan_fwd_noalloc(N.ptr(q), N.ptr(q), N.ptr(q), N.ptr(f), N.ptr(q), None, None,
                                       None, None, 4096, 1 << 20, 64, 64, N.BF16, N.BF16,
                                       N.stream_ptr(dev))
    assert st == N.ERR_TOO_LARGE
    assert b"16 MiB" in L.mogt_status_string(st)
    # arguments are checked before the shared array is touched
    st = L.mogt_gated_scan_fwd_noalloc(N.ptr(q), N.ptr(q), N.ptr(q), None, N.ptr(q), None, None,
                                       None, None, 1, 64, 64, 64, N.BF16, N.BF16, N.stream_ptr(dev))
    assert st == N.ERR_ARG
