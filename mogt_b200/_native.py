"""ctypes binding of libmogt_scan.so (the C ABI declared in include/mogt_scan.h).

The library is loaded on first use and the product path has no alternative:
if the shared object is missing, every op raises instead of computing
anything on the CPU.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmogt_scan.so"

F32, BF16, F16 = 0, 1, 2
MATRIX_FP32, MATRIX_TF32X3 = 0, 1
_DT = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

OK, ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_LAUNCH, ERR_TIMEOUT, ERR_WORKSPACE, ERR_UNSUPPORTED, ERR_ARG, ERR_TOO_LARGE = range(10)

_vp, _i64, _int, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t

# name -> (restype, argtypes); must match include/mogt_scan.h
SIGNATURES = {
    "mogt_abi_version": (_int, []),
    "mogt_status_string": (ctypes.c_char_p, [_int]),
    "mogt_workspace_status": (_int, [_vp, _vp, ctypes.POINTER(_int), ctypes.POINTER(ctypes.c_uint32)]),
    "mogt_workspace_clear": (_int, [_vp, _sz, _vp]),
    "mogt_gated_scan_num_chunks": (_i64, [_i64, _i64, _i64, _int]),
    "mogt_gated_scan_fwd_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _int]),
    "mogt_gated_scan_fwd": (_int, [_vp] * 9 + [_i64] * 4 + [_int, _int, _vp, _sz, _vp]),
    "mogt_gated_scan_fwd_resume": (_int, [_vp] * 9 + [_i64] * 4 + [_int, _int, _vp, _sz, _vp]),
    "mogt_gated_scan_fwd_noalloc": (_int, [_vp] * 9 + [_i64] * 4 + [_int, _int, _vp]),
    "mogt_gated_scan_fwd_noalloc_status": (_int, [_vp, ctypes.POINTER(_int), ctypes.POINTER(ctypes.c_uint32)]),
    "mogt_gated_scan_bwd_workspace_bytes": (_sz, [_i64] * 4 + [_int]),
    "mogt_gated_scan_bwd": (_int, [_vp] * 12 + [_i64] * 4 + [_int, _vp, _sz, _vp]),
    "mogt_matrix_scan_fwd": (_int, [_vp] * 8 + [_i64] * 3 + [_int, _int, _vp]),
    "mogt_matrix_scan_chunked_scratch_bytes": (_sz, [_i64] * 3),
    "mogt_matrix_scan_fwd_chunked": (_int, [_vp] * 8 + [_i64] * 3 + [_int, _int, _int] + [_vp, _vp, _sz, _vp]),
    "mogt_matrix_scan_bwd_scratch_bytes": (_sz, [_i64] * 3),
    "mogt_matrix_scan_bwd": (_int, [_vp] * 13 + [_i64] * 3 + [_int, _vp, _vp, _sz, _vp]),
    "mogt_diag_scan_norm_scratch_bytes": (_sz, [_i64] * 4 + [_int]),
    "mogt_diag_scan_norm_fwd": (_int, [_vp, _vp, _i64, ctypes.c_float, _vp, _vp, ctypes.c_float, _vp, _vp]
                                + [_i64] * 4 + [_int, _int, _vp, _vp, _sz, _vp]),
    "mogt_diag_scan_norm_bwd_scratch_bytes": (_sz, [_i64] * 4),
    "mogt_diag_scan_norm_bwd": (_int, [_vp, _vp, _i64, ctypes.c_float, _vp, ctypes.c_float, _vp, _vp, _vp, _vp,
                                       _vp, _vp] + [_i64] * 4 + [_int, _int, _vp, _vp, _sz, _vp]),
    "mogt_connection_map": (_int, [_vp, _vp, _i64, _i64, _int, _int, ctypes.c_float, ctypes.c_float, _int, _int, _vp]),
    "mogt_ce_rows_fwd": (_int, [_vp, _vp, _i64, _i64, _vp, _vp, _vp]),
    "mogt_ce_rows_bwd": (_int, [_vp, _vp, _vp, _i64, _i64, ctypes.c_float, _vp]),
    "mogt_affine_scan_workspace_bytes": (_sz, [_i64] * 4),
    "mogt_affine_scan_fwd": (_int, [_vp] * 4 + [_i64] * 4 + [_int] * 4 + [_vp, _sz, _vp]),
    "mogt_affine_grad_u": (_int, [_vp] * 3 + [_i64] * 4 + [_int, _vp]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """Load libmogt_scan.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m mogt_b200.build` "
                        "(the MOGT scan ops have no CPU fallback)")
                L = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                if L.mogt_abi_version() != 2:
                    raise RuntimeError("libmogt_scan.so ABI version mismatch")
                _lib = L
    return _lib


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}") from None


def check(status: int, what: str) -> None:
    if status == OK:
        return
    msg = lib().mogt_status_string(status).decode()
    if status in (ERR_SHAPE, ERR_DTYPE, ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg} (status {status})")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


# Device-side failures.  A look-back or mbarrier wait that gives up records
# MOGT_ERR_TIMEOUT in the 256-byte header of the call's workspace (the kernel
# then finishes with wrong results instead of hanging).  After every launch
# the ops below queue a 4-byte copy of that word into pinned host memory; the
# next call that uses the same workspace raises RuntimeError when the copy has
# landed and shows an error, so a failure surfaces without a host
# synchronisation on the hot path.  With MOGT_SYNC_CHECK=1 in the environment
# every call waits for its own result and raises at once; check_errors()
# waits and raises on demand.
import os

SYNC_CHECK = os.environ.get("MOGT_SYNC_CHECK", "0") not in ("", "0")


class DeviceTimeout(RuntimeError):
    """A bounded device-side wait gave up: the call's results are not valid."""


def _raise_timeout(what, unit):
    raise DeviceTimeout(f"{what}: a device-side wait timed out (unit {unit}); "
                        "the results of that call are not valid")


class _Workspace:
    __slots__ = ("buf", "slot", "event", "what", "tag")

    def __init__(self, buf):
        self.buf = buf
        self.slot = torch.zeros(2, dtype=torch.int32).pin_memory()
        self.event = None
        self.what = None
        self.tag = None   # what the last call left in the buffer (see ops.gated_scan_fwd)

    def clear_error(self):
        self.buf[12:20].zero_()
        self.slot.zero_()

    def poll(self):
        """Raise if an earlier call on this workspace recorded a timeout
        whose status copy has already arrived (no synchronisation)."""
        if self.event is not None and self.event.query():
            self.event = None
            err, unit = int(self.slot[0]), int(self.slot[1])
            if err:
                what = self.what
                self.clear_error()
                _raise_timeout(what, unit)

    def after_launch(self, what):
        self.what = what
        stream = torch.cuda.current_stream(self.buf.device)
        self.slot.copy_(self.buf[12:20].view(torch.int32), non_blocking=True)
        if SYNC_CHECK:
            stream.synchronize()
            self.event = None
            err, unit = int(self.slot[0]), int(self.slot[1])
            if err:
                self.clear_error()
                _raise_timeout(what, unit)
            return
        ev = torch.cuda.Event()
        ev.record(stream)
        self.event = ev


class _Workspaces:
    """One zero-initialised workspace per (device, stream, kernel family),
    grown on demand.

    The kernels leave a workspace ready for the next call, so it is zeroed
    only when (re)allocated.  Calls on one stream are ordered, which is what
    sharing a workspace requires.  Every kernel family has its own buffer:
    their layouts differ, and a family that reused another's buffer could
    read that family's state data as its flags."""

    def __init__(self):
        self._ws = {}

    def entry(self, device: torch.device, nbytes: int, family: str) -> _Workspace:
        key = (device.index, torch.cuda.current_stream(device).cuda_stream, family)
        w = self._ws.get(key)
        if w is None or w.buf.numel() < nbytes:
            if w is not None:
                w.poll()
            size = max(nbytes, 0 if w is None else int(w.buf.numel() * 1.5))
            # made outside inference mode: the buffers are updated in place by
            # later calls whatever mode those run in
            with torch.inference_mode(False):
                w = _Workspace(torch.zeros(size + 256, dtype=torch.uint8, device=device))
            self._ws[key] = w
        else:
            w.poll()
        return w

    def get(self, device: torch.device, nbytes: int, family: str = "misc") -> torch.Tensor:
        return self.entry(device, nbytes, family).buf

    def status(self, device: torch.device):
        """(err, unit) of every workspace on `device` (synchronises)."""
        out = []
        for (idx, s, _fam), w in self._ws.items():
            if idx != device.index:
                continue
            err, unit = ctypes.c_int(0), ctypes.c_uint32(0)
            check(lib().mogt_workspace_status(ptr(w.buf), ctypes.c_void_p(s), ctypes.byref(err),
                                              ctypes.byref(unit)), "mogt_workspace_status")
            out.append((err.value, unit.value))
        return out

    def check(self, device: torch.device):
        """Synchronise and raise DeviceTimeout if any workspace on `device`
        holds a recorded timeout (the record is cleared)."""
        torch.cuda.synchronize(device)
        for (idx, _s, _fam), w in self._ws.items():
            if idx != device.index:
                continue
            w.event = None
            err, unit = (int(x) for x in w.buf[12:20].view(torch.int32).tolist())
            if err:
                what = w.what or "mogt kernel"
                w.clear_error()
                _raise_timeout(what, unit)


workspaces = _Workspaces()


def workspace_errors(device=None):
    """Return the sticky device-side error codes recorded in this process's
    workspaces on `device` (0 = none).  Synchronises the device."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    return [e for e, _ in workspaces.status(device)]


def check_errors(device=None):
    """Wait for `device` and raise DeviceTimeout if a call recorded a
    device-side timeout since the last check."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    workspaces.check(device)
