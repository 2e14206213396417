#!/usr/bin/env python
"""Benchmark of the MOGT scan core on B200.

Workload (the scan-core metric at d768): the headed gated
scan forward, B=1 per GPU, H=12 heads of dk=dv=64, T=32768, bf16 q/k/v, fp32
gates, bf16 output, fp32 state.  A step is one forward over one batch.
Multi-GPU runs are replicas (each rank scans its own sequence; no collective
on the data path), so ``value`` is weak-scaling whole-job tokens/s.

    python bench.py [--gpus N --steps K --warmup W]        # this library
    python bench.py --impl reference ...                   # reference CPU path

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# algorithmic bytes per (token, head): q, k, v (3 x 64 bf16) + f (fp32) + o (64 bf16)
BYTES_PER_TOKEN_HEAD = 3 * 64 * 2 + 4 + 64 * 2
METRIC = "gated scan core forward throughput (d768: H=12, dk=dv=64, T=32768, bf16)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--T", type=int, default=32768)
    p.add_argument("--heads", type=int, default=12)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extra", action="store_true")
    p.add_argument("--profile-case", choices=sorted(PROFILE_CASES),
                   help="run one named workload three times on cuda:0 and exit (for ncu captures)")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_inputs(B, H, T, seed):
    import torch
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, T, 64, generator=g)
    k = torch.randn(B, H, T, 64, generator=g)
    k = k / k.norm(dim=-1, keepdim=True)
    v = torch.randn(B, H, T, 64, generator=g)
    f = torch.sigmoid(torch.randn(B, H, T, generator=g) + 2.0)
    return q.bfloat16(), k.bfloat16(), v.bfloat16(), f.float()


# ----------------------------------------------------------------------------
# CPU reference path: the oracle's restatement of the reference operator
# (affine_scan_sequential on U = f I, V = (1-f) k v^T, then the readout).
# ----------------------------------------------------------------------------
def cpu_reference_run(q, k, v, f, Ts, form="torch"):
    """Time the reference algorithm on the first Ts steps of every head.

    form "torch": the reference's own CPU code path restated in torch (the
    per-step bmm loop of affine_scan.py:47-55 on dense f*I transitions, fp32
    state, then the readout einsum), building U and V from q, k, v, f inside
    the timed region as the reference operator's caller does;
    form "numpy": the oracle's numpy restatement (U and V built outside)."""
    from oracle import scan_oracle as O
    qs, ks, vs, fs = (t[:, :, :Ts].float() for t in (q, k, v, f))
    if form == "torch":
        t0 = time.perf_counter()
        o = O.gated_scan_torch_reference_path(qs, ks, vs, fs)
        return time.perf_counter() - t0, o
    import numpy as np
    qs, ks, vs, fs = (t.numpy() for t in (qs, ks, vs, fs))
    B, H, _, d = qs.shape
    ff = fs.reshape(B * H, Ts).astype(np.float32)
    U = ff[..., None, None] * np.eye(d, dtype=np.float32)
    Vin = (1.0 - ff)[..., None, None] * (ks.reshape(B * H, Ts, d, 1) * vs.reshape(B * H, Ts, 1, d))
    qf = qs.reshape(B * H, Ts, d)
    t0 = time.perf_counter()
    S = O.affine_scan_sequential(U, Vin, state_dtype=np.float32, output_dtype=np.float32)
    o = np.einsum("ntkv,ntk->ntv", S, qf)
    return time.perf_counter() - t0, o


def cpu_threads():
    import torch
    return int(torch.get_num_threads())


def _sample(q, k, v, f, form, target_s):
    dt, _ = cpu_reference_run(q, k, v, f, 256, form)
    per_tok = max(dt / 256, 1e-6)
    Ts = int(min(q.shape[2], 4096, max(64, target_s / per_tok)))
    dt, _ = cpu_reference_run(q, k, v, f, Ts, form)
    return Ts, dt


def cpu_baseline_sample(q, k, v, f, target_s=12.0):
    """The reference's CPU path (torch form) on a bounded sample, and the
    numpy restatement beside it."""
    B = q.shape[0]
    Ts, dt = _sample(q, k, v, f, "torch", target_s)
    Tn, dtn = _sample(q, k, v, f, "numpy", target_s / 2)
    return {"value": B * Ts / dt, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
            "sample": f"first {Ts} of {q.shape[2]} steps, all {q.shape[1]} heads, B={B}: the reference's "
                      f"CPU code path (per-step torch.bmm loop of affine_scan_sequential on dense f*I, fp32, "
                      f"+ readout einsum) restated in torch; {dt:.1f} s",
            "numpy_port": {"value": B * Tn / dtn, "unit": "tokens/s",
                           "sample": f"first {Tn} steps, numpy restatement (oracle); {dtn:.1f} s"}}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    q, k, v, f = make_inputs(args.batch, args.heads, args.T, seed=0)
    dt, _ = cpu_reference_run(q, k, v, f, 256)
    per_tok = max(dt / 256, 1e-6)
    budget = 100.0  # seconds of CPU work for the whole --steps + --warmup run
    Ts = int(min(args.T, 4096, max(8, budget / (args.steps + args.warmup) / per_tok)))
    for _ in range(args.warmup):
        cpu_reference_run(q, k, v, f, Ts)
    t_total = 0.0
    for _ in range(args.steps):
        dt, _ = cpu_reference_run(q, k, v, f, Ts)
        t_total += dt
    value = args.batch * Ts * args.steps / t_total
    cores = cpu_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t_total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2_core_fwd", "B": args.batch, "H": args.heads, "T": args.T,
                   "dk": 64, "dv": 64, "sample_steps_per_step": Ts},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"each step: first {Ts} of {args.T} steps of all {args.heads} heads "
                                   "(the reference's CPU code path -- per-step torch.bmm loop of "
                                   "affine_scan_sequential on dense f*I, fp32 state, + readout -- "
                                   "restated in torch; the reference tree is not on the GPU box)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------
# clocks during the timed region (NVML polling thread)
# ----------------------------------------------------------------------------
class ClockSampler:
    def __init__(self, index):
        self.samples = []
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def sample(self, tag):
        if not self.ok:
            return
        nv = self.nv
        try:
            mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
            reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            self.samples.append((tag, time.perf_counter(), mhz, reasons))
        except Exception:
            pass

    def _loop(self):
        while not self._stop.is_set():
            self.sample("bg")
            time.sleep(0.002)

    def start(self):
        if self.ok:
            self.t = threading.Thread(target=self._loop, daemon=True)
            self.t.start()

    def stop(self):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self, t0, t1):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        nv = self.nv
        inside = [s for s in self.samples if t0 <= s[1] <= t1] or self.samples[-3:]
        names = {
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        mask = 0
        for s in inside:
            mask |= s[3]
        reasons = [n for n, bit in names.items() if mask & bit]
        return {"sm_mhz": statistics.median(s[2] for s in inside), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(inside)}


# One forward at the bench workload is three launches: gated_chunk_local,
# gated_seg_carry and gated_chunk_out (chained by programmatic dependent
# launch).  The roofline treats the three as the unit: achieved = algorithmic
# bytes / event time of the whole forward.  Traffic is their summed DRAM bytes
# (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu capture of each
# kernel without cache flushing, so that the output pass's L2 hits on what the
# local pass left behind count as they do in the timed loop; the command is in
# the forward's profile summary.  Updated by hand when the kernels change;
# None when no capture of the current kernels exists.
FWD_KERNELS = ("gated_chunk_local", "gated_seg_carry", "gated_chunk_out")
FWD_TRAFFIC_BYTES_PER_LAUNCH = 367570688


def measured_peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def run_b200(args):
    import torch
    import torch.distributed as dist

    import mogt_b200
    from mogt_b200 import _native, ops

    world, rank, local = dist_env()
    if world > 1:
        # what the C++ side prints (the communicator's NCCL version line among
        # it) goes to stderr: file descriptor 1 is pointed at stderr and Python's
        # stdout keeps a duplicate of the original, so stdout carries only the
        # JSON line
        sys.stdout.flush()
        out_fd = os.dup(1)
        os.dup2(2, 1)
        sys.stdout = os.fdopen(out_fd, "w", buffering=1)
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    B, H, T = args.batch, args.heads, args.T

    # two input sets (each > L2 at T=32768) alternated between steps
    host = make_inputs(B, H, T, seed=1000 + rank)
    sets = [tuple(t.to(dev) for t in host), tuple(t.to(dev) for t in make_inputs(B, H, T, seed=2000 + rank))]
    o_dev = [torch.empty(B, H, T, 64, dtype=torch.bfloat16, device=dev) for _ in sets]

    L = _native.lib()
    nbytes = L.mogt_gated_scan_fwd_workspace_bytes(B * H, T, 64, 64, _native.BF16)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        q, k, v, f = sets[i & 1]
        o = o_dev[i & 1]
        st = L.mogt_gated_scan_fwd(_native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(f),
                                   _native.ptr(o), None, None, None, None, B * H, T, 64, 64,
                                   _native.BF16, _native.BF16, _native.ptr(ws), nbytes,
                                   _native.ctypes.c_void_p(stream.cuda_stream))
        if st != 0:
            raise RuntimeError(f"mogt_gated_scan_fwd failed: {st}")

    clocks = ClockSampler(dev.index)
    clocks.start()
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.perf_counter()
    e0.record(stream)
    # clocks are sampled by the sampler's own thread only: a synchronous NVML
    # query here would stall the launches and leave the GPU idle inside the
    # timed region when few steps are queued
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    t_wall1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    errs = _native.workspace_errors(dev)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clocks.stop()
    ms_per_step = ms / args.steps
    tokens_per_step = B * T * world
    value = tokens_per_step / (ms_per_step / 1e3)

    # ---- end to end through the public API: host (pinned) -> device -> host ----
    # Every step copies its inputs from pinned host memory, runs
    # mogt_b200.gated_scan and copies the output back.  Steps are pipelined the
    # way a serving loop would run them: the device-to-host copy of step i runs
    # on a second stream while step i+1's host-to-device copy and scan run
    # (PCIe moves both directions at once); inputs and outputs are
    # double-buffered so no copy overwrites data still in use.
    hq, hk, hv, hf = (t.pin_memory() for t in host)
    ho = [torch.empty(B, H, T, 64, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    din = [tuple(torch.empty_like(t, device=dev) for t in host) for _ in range(2)]
    e2e_steps = max(3, min(args.steps, 20))
    s_out = torch.cuda.Stream(dev)
    keep = [None, None]

    def e2e_step(i):
        dq, dk, dv, df = din[i & 1]
        dq.copy_(hq, non_blocking=True)
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
        df.copy_(hf, non_blocking=True)
        o = mogt_b200.gated_scan(dq, dk, dv, df)
        done = torch.cuda.Event()
        done.record(stream)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            ho[i & 1].copy_(o, non_blocking=True)
        o.record_stream(s_out)
        keep[i & 1] = o

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    fin = torch.cuda.Event()
    fin.record(s_out)
    stream.wait_event(fin)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = tokens_per_step / (e2e_ms / e2e_steps / 1e3)
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = ho[0].numel() * ho[0].element_size()
    # parity spot-check of the e2e result against the device result
    ok = torch.equal(ho[(e2e_steps - 1) & 1].to(dev), o_dev[0])

    extra = {}
    if not args.no_extra:
        bb = extra_backbone(dev, world, rank)
        sp = extra_sp(dev, world, rank) if world > 1 else None
        if rank == 0:
            extra = extra_affine(dev)
            extra["backbone"] = bb
            extra["gated_bwd_config2"] = extra_backward(dev, B, H, T)
            extra["matrix_scan_config3"] = extra_matrix(dev)
            extra["config2_sweep"] = extra_config2_sweep(dev)
            extra["connection_map_backbone"] = extra_connection(dev)
            if sp is not None:
                extra["sequence_parallel_config5"] = sp

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(*host)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    peak, peak_kind = measured_peak_hbm()
    alg_bytes = BYTES_PER_TOKEN_HEAD * B * H * T
    achieved = alg_bytes / (ms_per_step / 1e3) / 1e9
    traffic = FWD_TRAFFIC_BYTES_PER_LAUNCH
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded q,k,v ~ N(0,1) (k L2-normalised), f = sigmoid(N(2,1))",
        "config": {"workload": "config2_core_fwd", "B": B, "H": H, "T": T, "dk": 64, "dv": 64,
                   "per_gpu": "independent sequence per rank (replicas)",
                   "l2": "2 input sets alternated, each 202.9 MB (> 126 MB L2)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "algorithmic_bytes_per_launch": alg_bytes,
                     "kernels": "+".join(FWD_KERNELS) + " (one forward)"},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps, "ms_per_step": e2e_ms / e2e_steps,
                "api": "mogt_b200.gated_scan", "matches_device_result": bool(ok),
                "pipelining": "copy-out of step i on a second stream overlaps step i+1's copy-in and scan"},
        "gpu_launches": args.steps * len(FWD_KERNELS),
        "clocks": clocks.summary(t_wall0, t_wall1),
        "workspace_errors": errs,
    }
    if extra:
        line["extra"] = extra
    print(json.dumps(line), flush=True)
    return 0


def extra_affine(dev):
    """Reference-native core shape (d768, r=16: U [1,L,16,16] fp32,
    V [1,L,16,48] fp32, H fp32) at L = 32768: the shape of the reference's
    published 5.48 ms (L4) Triton-hybrid number."""
    import torch
    from mogt_b200 import ops
    g = torch.Generator().manual_seed(7)
    Ls = 32768
    U = (torch.eye(16) + 0.01 * torch.randn(1, Ls, 16, 16, generator=g)).to(dev)
    V = torch.randn(1, Ls, 16, 48, generator=g).to(dev)
    for _ in range(5):
        ops.affine_scan(U, V)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 50
    e0.record()
    for _ in range(n):
        ops.affine_scan(U, V)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    alg = 7168 * Ls
    return {"affine_r16_c48_L32768": {"ms": ms, "GBps": alg / (ms / 1e3) / 1e9,
                                      "reference_L4_triton_hybrid_ms": 5.48,
                                      "note": "not L2-flushed (235 MB working set > L2)"}}


def extra_backward(dev, B, H, T):
    """BASELINE config 2, backward: the reverse-time chunked tensor-core
    kernel on the forward's bf16 chunk states (two input sets alternated,
    each > L2).  Algorithmic bytes per (token, head): q, k, v, f, do read
    (516) + dq, dk, dv, df written (388) = 904; the saved chunk states the
    kernel also reads (8192 / 64 = 128 B per token and head) are reported
    separately."""
    import torch
    from mogt_b200 import ops
    sets = []
    for seed in (3000, 4000):
        q, k, v, f = (t.to(dev) for t in make_inputs(B, H, T, seed))
        g = torch.randn(B, H, T, 64, generator=torch.Generator().manual_seed(seed)).to(dev).bfloat16()
        _, _, _, cs = ops.gated_scan_fwd(q, k, v, f, save_states=True)
        sets.append((q, k, v, f, g, cs))
    step = lambda i: ops.gated_scan_bwd(*sets[i & 1][:5], chunk_states=sets[i & 1][5])
    for i in range(4):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 20
    e0.record()
    for i in range(n):
        step(i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    alg = 904 * B * H * T
    return {"ms": ms, "tokens_per_s": B * T / (ms / 1e3), "GBps": alg / (ms / 1e3) / 1e9,
            "algorithmic_bytes": alg, "chunk_state_bytes": 128 * B * H * T,
            "dtype": "bf16 inputs, fp32 state/accumulate",
            "note": "includes the Python-side output allocation; forward with saved chunk states not timed"}


def extra_sp(dev, world, rank):
    """one sequence of T = 262144 (B=1, H=12, 64x64) split
    into contiguous segments over the ranks; segment carries all-gathered over
    NCCL, local correction scan.  Time = max over ranks; whole-job tokens/s."""
    import torch
    import torch.distributed as dist
    from mogt_b200.sp import gated_scan_sp
    T = 262144
    T_loc = T // world
    q, k, v, f = (t.to(dev) for t in make_inputs(1, 12, T_loc, 5000 + rank))
    run = lambda: gated_scan_sp(q, k, v, f)
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 10
    e0.record()
    for _ in range(n):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # parity: the joined segments against a one-GPU scan of the whole sequence
    # (rank 0 regenerates every rank's seeded segment)
    o = run()
    outs = [torch.empty_like(o) for _ in range(world)]
    dist.all_gather(outs, o)
    err = None
    if rank == 0:
        from mogt_b200 import ops
        segs = [tuple(t_.to(dev) for t_ in make_inputs(1, 12, T_loc, 5000 + r)) for r in range(world)]
        full = [torch.cat([sg[i] for sg in segs], 2) for i in range(4)]
        ref, _, _, _ = ops.gated_scan_fwd(*full)
        joined = torch.cat(outs, 2)
        err = float((joined.float() - ref.float()).abs().max() / ref.float().abs().max())
        del segs, full, ref, joined
    del outs
    torch.cuda.empty_cache()
    return {"ms": ms, "tokens_per_s": T / (ms / 1e3), "T": T, "ranks": world,
            "rel_max_err_vs_one_gpu_scan": err,
            "note": "state-only segment scan + NCCL all-gather of (decay, state) carries + the forward "
                    "resumed from the incoming state (carry + output pass); outputs bf16 on both sides"}


def _time_call(call, n, warm=2):
    import torch
    for _ in range(warm):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        call()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / n


def extra_matrix(dev):
    """dense Cayley transitions, B=2, H=8, T=8192, d=64,
    bf16 q/k/v, fp32 A.  Forward: minimal flops per (step, head) 2*64^3 +
    2*64^2 + 2*64^2 = 540,672 and bytes 16,900 (A 16384 + q,k,v 384 + f 4 +
    o 128).  Backward: bytes per (step, head) A 16384 read + dA 16384 written
    + q,k,v,do,f read (516) + dq,dk,dv,df written (388) = 33,672; minimal
    flops 3 * 2 * 64^3 (state recompute, adjoint carry, dA) = 1,572,864."""
    import torch
    from mogt_b200 import ops
    B, H, T, d = 2, 8, 8192, 64
    A = _cayley_transitions(B, H, T, d, dev, 11)
    g = torch.Generator(device=dev).manual_seed(12)
    q, k, v = (torch.randn(B, H, T, d, generator=g, device=dev).bfloat16() for _ in range(3))
    f = torch.sigmoid(torch.randn(B, H, T, generator=g, device=dev) + 2.0)
    units = B * H * T
    out = {}
    for prec in ("fp32", "tf32x3"):
        ms = _time_call(lambda: ops.matrix_scan_fwd(A, q, k, v, f, precision=prec), 3)
        out[f"fwd_{prec}"] = {"ms": ms, "TFLOPs": units * 540672 / (ms / 1e3) / 1e12,
                              "GBps": units * 16900 / (ms / 1e3) / 1e9}
    out["fwd_fp32"]["note"] = ("default: chunked, per-chunk [P | S_loc] with fp32 FMAs (round-to-nearest), "
                               "carries per head, outputs per chunk; within 1e-5 of the fp64 oracle at T=8192")
    out["fwd_tf32x3"]["note"] = ("opt-in tensor-core form (3xTF32 tcgen05); its accumulation bias reaches "
                                 "4e-4 relative at T=8192, above the 1e-4 fp32 bar")
    do = torch.randn(B, H, T, d, generator=g, device=dev).bfloat16()
    _, _, saved = ops.matrix_scan_fwd(A, q, k, v, f, save_for_backward=True)
    ms = _time_call(lambda: ops.matrix_scan_bwd(A, q, k, v, f, do, saved), 2, warm=1)
    out["bwd"] = {"ms": ms, "TFLOPs": units * 1572864 / (ms / 1e3) / 1e12,
                  "GBps": units * 33672 / (ms / 1e3) / 1e9,
                  "note": "reverse-time chunked on the forward's saved chunk states, fp32 FMAs; "
                          "includes the Python-side output allocation"}
    del A, saved
    torch.cuda.empty_cache()
    return out


def extra_connection(dev):
    """Connection map at the backbone shape (B=8, L=32768, r=16; one layer):
    the kernel against torch.matrix_exp (what the reference calls,
    model_mogt.py:85) on the same GPU.  Bytes per token: M bf16 512 + U bf16
    512."""
    import torch
    from mogt_b200.connection import connection_map
    g = torch.Generator(device=dev).manual_seed(3)
    M = (0.05 * torch.randn(8, 32768, 16, 16, generator=g, device=dev)).bfloat16()
    out = {}
    for impl in ("matrix_exp", "cayley"):
        ms = _time_call(lambda: connection_map(M, impl), 5)
        out[impl] = {"ms": ms, "matrices_per_s": M.numel() / 256 / (ms / 1e3)}

    def torch_expm():
        A = (M - M.transpose(-1, -2)).float() / 16
        return (torch.matrix_exp(A) * 0.999).to(M.dtype)
    out["torch_matrix_exp_ms"] = _time_call(torch_expm, 3)
    return out


def extra_config2_sweep(dev):
    """BASELINE config 2 at T = 8192 and 16384 (the bench line is T = 32768):
    forward and backward timed separately, 516 / 904 algorithmic bytes per
    (token, head).  The forward is timed through the C ABI with preallocated
    buffers, as the bench line is (the Python wrapper's per-call host work
    would otherwise set the pace at these sizes); the backward through
    mogt_b200.ops (its output allocation included)."""
    from mogt_b200 import _native, ops
    import torch
    L = _native.lib()
    out = {}
    for T in (8192, 16384):
        q, k, v, f = (t.to(dev) for t in make_inputs(1, 12, T, 7000 + T))
        o = torch.empty(1, 12, T, 64, dtype=torch.bfloat16, device=dev)
        nbytes = L.mogt_gated_scan_fwd_workspace_bytes(12, T, 64, 64, _native.BF16)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        stream = _native.ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)

        def fwd():
            st = L.mogt_gated_scan_fwd(_native.ptr(q), _native.ptr(k), _native.ptr(v), _native.ptr(f),
                                       _native.ptr(o), None, None, None, None, 12, T, 64, 64,
                                       _native.BF16, _native.BF16, _native.ptr(ws), nbytes, stream)
            if st != 0:
                raise RuntimeError(f"mogt_gated_scan_fwd failed: {st}")
        ms_f = _time_call(fwd, 50, warm=5)
        g = torch.randn(1, 12, T, 64, generator=torch.Generator().manual_seed(T)).to(dev).bfloat16()
        _, _, _, cs = ops.gated_scan_fwd(q, k, v, f, save_states=True)
        ms_b = _time_call(lambda: ops.gated_scan_bwd(q, k, v, f, g, chunk_states=cs), 20)
        out[f"T{T}"] = {"fwd_ms": ms_f, "fwd_tokens_per_s": T / (ms_f / 1e3),
                        "fwd_GBps": 516 * 12 * T / (ms_f / 1e3) / 1e9,
                        "bwd_ms": ms_b, "bwd_GBps": 904 * 12 * T / (ms_b / 1e3) / 1e9}
        del ws, o
    return out


def extra_backbone(dev, world, rank):
    """MOGT backbone forward (d768, 4 layers, r=16, vocab
    32000, identity connection + rank-wise coupled gate), T=32768, bf16
    autocast, global batch 8 split over the ranks, random N(0, 0.02) weights;
    whole-job tokens/s with the time taken as the max over ranks."""
    import torch
    import torch.distributed as dist
    from mogt_b200.backbone import MOGTModel, configure_identity_coupled
    T, layers, global_b = 32768, 4, 8
    b_local = max(1, global_b // world)
    torch.manual_seed(1234 + rank)
    model = MOGTModel(32000, 768, layers, 16)
    for p in model.parameters():
        torch.nn.init.normal_(p, std=0.02)
    configure_identity_coupled(model)
    model = model.to(dev).eval()
    ids = torch.randint(0, 32000, (b_local, T), device=dev)
    def run():
        with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
            return model(ids)
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 3
    e0.record()
    for _ in range(n):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del model
    torch.cuda.empty_cache()
    return {"tokens_per_s": b_local * world * T / (ms / 1e3), "ms_per_step": ms,
            "config": f"d768 r16 4 layers vocab 32000, B={b_local}/GPU x {world}, T={T}, bf16 autocast",
            "reference_L4_2layer_B1_tokens_per_s": 422000}


def _cayley_transitions(B, H, T, d, dev, seed):
    """Config-3 transitions A_t = solve(I - W_t, I + W_t), W_t = 0.05 (M - M^T)."""
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    M = torch.randn(B, H, T, d, d, generator=g, device=dev)
    W = 0.05 * (M - M.transpose(-1, -2))
    I = torch.eye(d, device=dev)
    return torch.linalg.solve(I - W, I + W).contiguous()


def _case_fwd_config2(dev):
    from mogt_b200 import ops
    q, k, v, f = (t.to(dev) for t in make_inputs(1, 12, 32768, 0))
    return lambda: ops.gated_scan_fwd(q, k, v, f)


def _case_bwd_config2(dev):
    import torch
    from mogt_b200 import ops
    q, k, v, f = (t.to(dev) for t in make_inputs(1, 12, 32768, 0))
    g = torch.randn(1, 12, 32768, 64, device=dev).bfloat16()
    _, _, _, cs = ops.gated_scan_fwd(q, k, v, f, save_states=True)
    return lambda: ops.gated_scan_bwd(q, k, v, f, g, chunk_states=cs)


def _case_matrix(B, H, T):
    def make(dev):
        import torch
        from mogt_b200 import ops
        A = _cayley_transitions(B, H, T, 64, dev, 11)
        g = torch.Generator(device=dev).manual_seed(12)
        q, k, v = (torch.randn(B, H, T, 64, generator=g, device=dev).bfloat16() for _ in range(3))
        f = torch.sigmoid(torch.randn(B, H, T, generator=g, device=dev) + 2.0)
        return lambda: ops.matrix_scan_fwd(A, q, k, v, f)
    return make


def _case_diag(B, L):
    def make(dev):
        import torch
        from mogt_b200 import ops
        g = torch.Generator(device=dev).manual_seed(0)
        V = torch.randn(B, L, 16, 48, generator=g, device=dev).bfloat16()
        z = torch.sigmoid(torch.randn(B, L, 16, 1, generator=g, device=dev) - 2.0)
        w = torch.ones(768, device=dev)
        return lambda: ops.diag_scan_norm(V, z, w, output_dtype=torch.bfloat16)
    return make


def _case_matrix_bwd(B, H, T):
    def make(dev):
        import torch
        from mogt_b200 import ops
        A = _cayley_transitions(B, H, T, 64, dev, 11)
        g = torch.Generator(device=dev).manual_seed(12)
        q, k, v, do = (torch.randn(B, H, T, 64, generator=g, device=dev).bfloat16() for _ in range(4))
        f = torch.sigmoid(torch.randn(B, H, T, generator=g, device=dev) + 2.0)
        _, _, saved = ops.matrix_scan_fwd(A, q, k, v, f, save_for_backward=True)
        return lambda: ops.matrix_scan_bwd(A, q, k, v, f, do, saved)
    return make


def _case_affine(B, L, C):
    def make(dev):
        import torch
        from mogt_b200 import ops
        g = torch.Generator().manual_seed(7)
        U = (torch.eye(16) + 0.01 * torch.randn(B, L, 16, 16, generator=g)).to(dev)
        V = torch.randn(B, L, 16, C, generator=g).to(dev)
        return lambda: ops.affine_scan(U, V)
    return make


# name -> builder of a zero-argument call; each case runs the call three times
PROFILE_CASES = {
    "fwd_config2": _case_fwd_config2,                 # gated forward, B=1 H=12 T=32768
    "bwd_config2": _case_bwd_config2,                 # gated backward on saved chunk states
    "matrix_config3": _case_matrix(2, 8, 8192),       # dense transitions, A = 2.2 GB
    "matrix_small": _case_matrix(1, 16, 2048),        # 512 chunk CTAs, A = 537 MB
    "diag_backbone": _case_diag(8, 32768),            # fused diagonal scan + norm, backbone shape
    "diag_small": _case_diag(8, 16384),
    "matrix_bwd_config3": _case_matrix_bwd(2, 8, 8192),  # dense-transition backward, A + dA = 4.3 GB
    "matrix_bwd_small": _case_matrix_bwd(1, 16, 2048),
    "affine_r16_c48": _case_affine(1, 32768, 48),        # reference-shape dense scan, 235 MB
    "affine_backbone": _case_affine(8, 32768, 48),
}


def run_profile_case(name):
    import torch
    dev = torch.device("cuda", 0)
    call = PROFILE_CASES[name](dev)
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    print(f"profile case {name}: 3 calls done")
    return 0


def main():
    args = parse()
    if args.profile_case:
        return run_profile_case(args.profile_case)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
