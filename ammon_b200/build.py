"""Builds libammon_b200.so (all CUDA sources for sm_100a with nvcc, host C++ with the host
compiler) in-tree.

Usage: python -m ammon_b200.build [--force] [-j N]
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
LIB = os.path.join(HERE, "libammon_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC,
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


# host-only C++ (the tokenizer) is compiled by the host compiler
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC]


def cuda_include() -> str:
    return os.path.join(os.path.dirname(os.path.dirname(nvcc())), "include")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(INCLUDE, "ammon_b200.h"))
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, obj, extra):
    if src.endswith(".cpp"):
        cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
        cmd = [cxx] + CXX_FLAGS + ["-I", cuda_include(), "-c", src, "-o", obj]
    else:
        cmd = [nvcc()] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compiler failed on {os.path.basename(src)}:\n{r.stderr}")
    return r.stderr


def build(force: bool = False, jobs: int = 0, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = headers()
    objs, todo = [], []
    for src in sources():
        obj = os.path.join(BUILD, os.path.splitext(os.path.basename(src))[0] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            todo.append((src, obj))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(jobs) as ex:
            futs = {ex.submit(_compile, s, o, extra): s for s, o in todo}
            for f in cf.as_completed(futs):
                log = f.result()
                if verbose_ptxas and log:
                    sys.stderr.write(log)
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.j, a.ptxas_verbose))


if __name__ == "__main__":
    main()
