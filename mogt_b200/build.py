"""Build libmogt_scan.so in-tree with nvcc for sm_100a.

    python -m mogt_b200.build          # or __graft_entry__.build()

Each ``csrc/*.cu`` is compiled to an object (``-Xcompiler -fPIC``) under
``mogt_b200/_build`` and the objects are linked into
``mogt_b200/lib/libmogt_scan.so`` (CUDA runtime linked statically, so the
library does not depend on which libcudart the host process loaded).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libmogt_scan.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
         f"-I{PKG.parent / 'include'}"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmogt_scan.so")
    return cand


def build(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted((PKG.parent / "include").glob("*.h"))
    newest_hdr = max((h.stat().st_mtime for h in headers), default=0.0)
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if (not force and obj.exists() and obj.stat().st_mtime >= src.stat().st_mtime
                and obj.stat().st_mtime >= newest_hdr):
            continue
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        log = BUILD / (src.stem + ".ptxas.txt")
        log.write_text(res.stdout + res.stderr)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError(f"nvcc failed on {src.name}")
        if verbose:
            sys.stdout.write(res.stderr)
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-cudart", "static"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link of libmogt_scan.so failed")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
