"""Sequence-parallel protocol on CPU ranks (gloo, world sizes 2 and 3).

The collective logic of mogt_b200.sp.gated_scan_sp (segment carry ->
all-gather -> carry combine -> local scan from the incoming state) is run
with the oracle as the local scan, so it needs no GPU; the CUDA local scan is
covered by the GPU tests.  Failure detection: a rank that leaves before the
exchange makes the others' collective fail with an error instead of hanging.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_fwd(q, k, v, f, *, initial_state=None, output_dtype=None, want_final=False,
                want_output=True, save_states=False):
    from oracle import scan_oracle as O
    S0 = None if initial_state is None else initial_state.double().numpy()
    o, S = O.gated_scan(q.double().numpy() if q is not None else k.double().numpy(),
                        k.double().numpy(), v.double().numpy(), f.double().numpy(), S0=S0,
                        return_final=True)
    dec = np.prod(f.double().numpy(), axis=-1)
    return (torch.from_numpy(o) if want_output else None,
            torch.from_numpy(S) if want_final else None,
            torch.from_numpy(dec) if want_final else None, None)


def _inputs(T, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, 2, T, 8, generator=g, dtype=torch.float64)
    k = torch.randn(1, 2, T, 8, generator=g, dtype=torch.float64)
    k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(1, 2, T, 8, generator=g, dtype=torch.float64)
    f = torch.sigmoid(torch.randn(1, 2, T, generator=g, dtype=torch.float64) + 2.0)
    S0 = torch.randn(1, 2, 8, 8, generator=g, dtype=torch.float64)
    return q, k, v, f, S0


def _worker(rank, world, port, T, out_q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    from mogt_b200.sp import gated_scan_sp
    q, k, v, f, S0 = _inputs(T)
    seg = T // world
    sl = slice(rank * seg, (rank + 1) * seg)
    if rank == fail_rank:
        os._exit(0)  # leaves before the exchange, between steps
    try:
        o = gated_scan_sp(q[:, :, sl], k[:, :, sl], v[:, :, sl], f[:, :, sl], initial_state=S0,
                          local_fwd=_oracle_fwd)
        out_q.put((rank, "ok", o.numpy()))
    except Exception as exc:  # the collective reports the missing peer
        out_q.put((rank, "error", repr(exc)))
    dist.destroy_process_group() if fail_rank is None else None


def _run(world, T, fail_rank=None):
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, q_out, fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    n_expect = world - (fail_rank is not None)
    res = [q_out.get(timeout=120) for _ in range(n_expect)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(res, key=lambda r: r[0])


@pytest.mark.parametrize("world", [2, 3])
def test_sp_matches_single_sequence_scan(world):
    from oracle import scan_oracle as O
    T = 60
    res = _run(world, T)
    assert all(r[1] == "ok" for r in res), res
    o = np.concatenate([r[2] for r in res], axis=2)
    q, k, v, f, S0 = _inputs(T)
    ref = O.gated_scan(q.numpy(), k.numpy(), v.numpy(), f.numpy(), S0=S0.numpy())
    assert np.abs(o - ref).max() < 1e-10


def test_sp_missing_rank_raises_instead_of_hanging():
    res = _run(2, 40, fail_rank=1)
    assert len(res) == 1 and res[0][0] == 0
    assert res[0][1] == "error"


def test_combine_carries_matches_sequential_composition():
    from mogt_b200.sp import combine_carries
    g = torch.Generator().manual_seed(1)
    world, B, H, d = 4, 1, 2, 3
    gathered = torch.randn(world, B, H, 1 + d * d, generator=g)
    X0 = torch.randn(B, H, d, d, generator=g)
    X = X0.clone()
    for r in range(3):
        A = gathered[r, :, :, 0].view(B, H, 1, 1)
        X = A * X + gathered[r, :, :, 1:].view(B, H, d, d)
    assert torch.allclose(combine_carries(gathered, 3, d, d, X0), X)
    assert torch.equal(combine_carries(gathered, 0, d, d), torch.zeros(B, H, d, d))
