"""Build the sm_100a decode library in-tree.

    python mamba3-fused-triton-kernel_b200/build_native.py [--ptxas-verbose] [--force]

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` (one process per file,
in parallel) and links ``lib/libmamba3_b200.so`` with the CUDA runtime linked
statically, so the library only needs the driver at run time.  Objects go to
``_build/`` next to this file.  A file is rebuilt when it or any header under
``csrc/`` / the repository ``include/`` is newer than its object.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
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
LIB = os.path.join(LIBDIR, "libmamba3_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
          "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(nvcc: str, src: str, obj: str, ptxas_verbose: bool) -> str:
    cmd = [nvcc, *ARCH, *CFLAGS, "-c", src, "-o", obj]
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr if ptxas_verbose else ""


def build(force: bool = False, ptxas_verbose: bool = False, jobs: int = 0) -> str:
    """Compile and link; returns the path of the shared library."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    hdr = _headers_mtime()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    todo, objs = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or ptxas_verbose or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr):
            todo.append((s, o))
    logs = []
    if todo:
        n = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=n) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, ptxas_verbose) for s, o in todo]
            for f in futs:
                logs.append(f.result())
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if ptxas_verbose:
        sys.stderr.write("".join(logs))
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    a = ap.parse_args()
    print(build(force=a.force, ptxas_verbose=a.ptxas_verbose, jobs=a.jobs))


if __name__ == "__main__":
    main()
