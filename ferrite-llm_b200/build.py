"""Builds libferrite_b200.so (sm_100a) in-tree with nvcc.

Usage: python ferrite-llm_b200/build.py [--force] [--jobs N]
Objects go to ferrite-llm_b200/_build/ (git-ignored); the shared library is
written next to this file so it travels with the source tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "libferrite_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Werror", "cross-execution-space-call",
          "-I", CSRC, "-I", INCLUDE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def host_cc() -> list[str]:
    # the image exports CC=/opt/gcc/bin/gcc; nvcc needs a complete host g++
    for cand in ("/usr/bin/g++",):
        if os.path.exists(cand):
            return ["-ccbin", cand]
    return []


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def headers_mtime() -> float:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(INCLUDE, "ferrite_b200.h"))
    return max(os.path.getmtime(h) for h in hs)


def compile_one(src: str, force: bool, extra: list[str]) -> str:
    obj = os.path.join(BUILD, src + ".o")
    srcp = os.path.join(CSRC, src)
    if not force and os.path.exists(obj):
        if os.path.getmtime(obj) >= max(os.path.getmtime(srcp), headers_mtime()):
            return obj
    cmd = [nvcc(), *host_cc(), *ARCH, *COMMON, *extra]
    if src.endswith(".cpp"):
        cmd += ["-x", "cu"]
    cmd += ["-c", srcp, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int = 0, extra: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    extra = extra or []
    jobs = jobs or min(8, os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force, extra), sources()))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc(), *host_cc(), *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    print(build(force=a.force or a.ptxas_verbose, jobs=a.jobs, extra=extra))
