"""Build libq8cuda.so in-tree for sm_100a (B200) with nvcc.

    python -m lama32_mojo_b200.build [--force] [-v]

Compiles every ``csrc/*.cu`` / ``*.cpp`` to an object under ``_build/`` and
links ``lama32_mojo_b200/libq8cuda.so`` against NCCL (the wheel-provided
libnccl.so.2 that torch also loads, found via rpath).  Rebuilds only stale
objects.  No JIT cache is involved, so the built library travels with the tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(REPO, "_build", "q8cuda")
LIB = os.path.join(PKG, "libq8cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nccl_dirs():
    """(include, lib) of the NCCL that torch ships (nvidia-nccl wheel), else system."""
    try:
        import nvidia.nccl as nn  # type: ignore
        base = os.path.dirname(nn.__file__) if getattr(nn, "__file__", None) else list(nn.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")) and glob.glob(os.path.join(lib, "libnccl.so*")):
            return inc, lib
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def _flags():
    inc, _ = _nccl_dirs()
    return ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", inc,
                   "-I", os.path.join(REPO, "include"), "--expt-relaxed-constexpr"]


def _stale(obj, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra=()):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        [os.path.join(REPO, "include", "q8cuda.h")]
    flags = _flags() + list(extra)
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            jobs.append([NVCC] + flags + ["-c", s, "-o", o])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for err in ex.map(run, jobs):
            if verbose and err.strip():
                print(err)
    if jobs or not os.path.exists(LIB) or _stale(LIB, objs):
        _, nlib = _nccl_dirs()
        link = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + [
            "-L", nlib, "-l:libnccl.so.2", "-Xlinker", "-rpath," + nlib, "-lcudart"]
        run(link)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra=extra))


if __name__ == "__main__":
    sys.exit(main())
