"""Builds libadamw4bit_b200.so (sm_100a) in-tree with nvcc.

    python -m adamw4bit_b200.build [--verbose-ptxas]

Every .cu file under csrc/ is compiled for sm_100a only (no PTX fallback) with
IEEE float semantics (--fmad=false, no fast-math), then linked into one shared
library next to this file, which the package loads with ctypes.  The CUDA
runtime is linked statically so the library does not depend on the runtime
torch ships.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
BUILD = os.path.join(ROOT, "_build")
LIB_NAME = "libadamw4bit_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-ffp-contract=off", "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose_ptxas: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(ROOT, "include", "adamw4bit_b200.h"))
    objs = []
    jobs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
        objs.append(obj)
        if force or verbose_ptxas or _stale(obj, [src, *headers, __file__]):
            cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
            if verbose_ptxas:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for cmd, r in ex.map(run, jobs):
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError(f"nvcc failed: {' '.join(cmd)}")
            if verbose_ptxas:
                sys.stderr.write(r.stderr)
    if force or _stale(LIB_PATH, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB_PATH, *objs, "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose_ptxas=a.verbose_ptxas, force=a.force))
