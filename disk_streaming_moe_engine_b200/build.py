"""Builds libdismoen_cuda.so in-tree for sm_100a with nvcc (no JIT cache, no torch).

    python -m disk_streaming_moe_engine_b200.build

Objects go to disk_streaming_moe_engine_b200/_build/, the library to
disk_streaming_moe_engine_b200/libdismoen_cuda.so.  A source newer than its object is
recompiled; the compiles run in parallel.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
BUILD = os.path.join(PKG_DIR, "_build")
LIB_PATH = os.path.join(PKG_DIR, "libdismoen_cuda.so")
INCLUDE = os.path.join(REPO_DIR, "include")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_LIB = "/usr/local/cuda/lib64"
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-diag-suppress", "177"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libdismoen_cuda.so")


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return max(os.path.getmtime(p) for p in paths)


def build(verbose: bool = False, force: bool = False, extra_flags: list[str] | None = None) -> str:
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    hdr = _headers_mtime()
    jobs = []
    objs = []
    for src in _sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr):
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *(extra_flags or []), "-I", INCLUDE, "-c", src, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for out in ex.map(run, jobs):
            if verbose and out.strip():
                print(out)
    if jobs or not os.path.exists(LIB_PATH):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", LIB_PATH, *objs, "-lcudart",
               "-Xlinker", "-rpath," + CUDA_LIB]
        run(cmd)
    return LIB_PATH


def build_oracle(verbose: bool = False) -> str:
    """Builds the CPU oracle (test infrastructure) with its Makefile."""
    oracle_dir = os.path.join(REPO_DIR, "oracle")
    r = subprocess.run(["make", "-C", oracle_dir], capture_output=True, text=True)
    if verbose:
        print(r.stdout, r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return os.path.join(oracle_dir, "liboracle.so")


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv, force="--force" in sys.argv)
    print(path)
