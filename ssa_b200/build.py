"""Build the sm_100a kernel library `ssa_b200/libssa_b200.so` in-tree.

    python -m ssa_b200.build [--force]

Each .cu file is compiled by nvcc for `-gencode arch=compute_100a,code=sm_100a`
(in parallel), then linked into one shared library with the static CUDA
runtime. The library exports only the C ABI of include/ssa_b200.h.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ_DIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libssa_b200.so")
SOURCES = ["ssa_graph.cu", "ssa_select_tc.cu", "ssa_hash_tc.cu", "ssa_select_rows.cu", "ssa_attn.cu", "ssa_capi.cu"]
HEADERS = ["ssa_common.cuh", "ssa_internal.h", "ssa_select_common.cuh", "ssa_tcgen05.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "ssa_b200.h")]
    jobs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ_DIR, src.replace(".cu", ".o"))
        if force or _stale(o, [s] + hdrs):
            jobs.append((s, o))

    def compile_one(job):
        s, o = job
        cmd = [nvcc()] + ARCH + FLAGS + ["-c", s, "-o", o + ".tmp"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {s}:\n{r.stderr}")
        os.replace(o + ".tmp", o)
        if verbose:
            print("compiled", os.path.basename(s))

    with ThreadPoolExecutor(max_workers=len(jobs) or 1) as ex:
        list(ex.map(compile_one, jobs))
    objs = [os.path.join(OBJ_DIR, s.replace(".cu", ".o")) for s in SOURCES]
    if force or jobs or _stale(LIB, objs):
        tmp = LIB + f".tmp{os.getpid()}"
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, LIB)
        if verbose:
            print("linked", LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=True))


if __name__ == "__main__":
    sys.exit(main())
