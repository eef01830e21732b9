"""Build libgdn_b200.so (the C-ABI kernel library) in-tree for sm_100a.

    python nano-vllm-extend_b200/build.py [--force] [-v]

Each csrc/*.cu is compiled to an object with nvcc (-gencode
arch=compute_100a,code=sm_100a -lineinfo -O3) and the objects are linked into
``lib/libgdn_b200.so`` next to this file.  Objects are rebuilt only when a
source or header is newer than them.  The library links the CUDA runtime
statically (no torch, no libcuda link dependency), so any process that has a
CUDA driver can dlopen it.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libgdn_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", "-I", CSRC, "-I", INCLUDE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    """Compile and link; returns the library path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    cc = nvcc()
    headers = _headers()
    flags = NVCC_FLAGS + list(extra_flags or [])
    jobs, objs = [], []
    for src in _sources():
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src[:-3] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers + [__file__]):
            jobs.append([cc] + flags + ["-c", s, "-o", o])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{p.stdout}\n{p.stderr}")
        if verbose and (p.stdout or p.stderr):
            print(p.stdout + p.stderr, flush=True)

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        run([cc] + ARCH + ["-shared", "-o", tmp] + objs + ["-cudart", "static"])
        os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v (regs/spills)")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_info else None
    print(build(force=a.force or a.ptxas_info, verbose=a.verbose or a.ptxas_info,
                extra_flags=extra))


if __name__ == "__main__":
    sys.exit(main())
