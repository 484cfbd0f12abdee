"""Builds libdbl_gdn2.so (the C-ABI library) in-tree with nvcc for sm_100a.

The library carries every CUDA kernel of the GDN-2 hot path and the ``extern "C"`` entry points
declared in ``include/dbl_gdn2.h``.  It links the CUDA runtime statically and has no torch
dependency, so any host (Rust FFI, C, Python ctypes) can load it.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libdbl_gdn2.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", f"-I{os.path.join(ROOT, 'include')}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the GDN-2 CUDA library cannot be built")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps() -> list[str]:
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hdrs.append(os.path.join(ROOT, "include", "dbl_gdn2.h"))
    return hdrs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/*.cu (in parallel) and link libdbl_gdn2.so.  Returns the library path."""
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    hdrs = _deps()
    objs = []
    jobs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            jobs.append([cc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            results = list(ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs))
        errors = [(c, r) for c, r in zip(jobs, results) if r.returncode != 0]
        for c, r in zip(jobs, results):
            if verbose or r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
        if errors:
            raise RuntimeError("nvcc failed for: " + ", ".join(os.path.basename(c[-3]) for c, _ in errors))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        r = subprocess.run([cc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs],
                           capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("linking libdbl_gdn2.so failed")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
