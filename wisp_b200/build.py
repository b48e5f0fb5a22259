"""Build ``wisp_b200/lib/libwisp_b200.so`` from ``wisp_b200/csrc`` with nvcc.

sm_100a only (B200).  The library links the CUDA runtime statically and
reaches no driver symbol at load time, so it also loads (for symbol checks)
on a machine without a GPU.

    python -m wisp_b200.build          # incremental
    python -m wisp_b200.build --force
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libwisp_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "-Xcompiler", "-Wall", "-diag-suppress", "177"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build wisp_b200")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    objdir = os.path.join(LIBDIR, "_obj")
    os.makedirs(objdir, exist_ok=True)
    nvcc = _nvcc()
    cmds, objs = [], []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src).replace(".cu", ".o"))
        cmd = [nvcc, *ARCH, *FLAGS, "-I", INCLUDE, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        cmds.append(cmd)
        objs.append(obj)
    # one nvcc per translation unit, in parallel
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as pool:
        for r in pool.map(lambda c: subprocess.run(c, capture_output=not verbose, text=True), cmds):
            if r.returncode:
                sys.stderr.write((r.stdout or "") + (r.stderr or ""))
                raise subprocess.CalledProcessError(r.returncode, r.args)
    tmp = LIB + ".tmp"
    subprocess.run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    sys.exit(0)
