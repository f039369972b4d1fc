"""Build recipe for libqgmoe.so (sm_100a only).

Compiles every csrc/*.cu with nvcc for `-gencode arch=compute_100a,code=sm_100a`
and links one shared library in-tree at qwen-go_b200/lib/libqgmoe.so, so the
built file travels with the source tree.  Objects go to qwen-go_b200/_build/.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(PKG_DIR, "csrc")
BUILD = os.path.join(PKG_DIR, "_build")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB = os.path.join(LIB_DIR, "libqgmoe.so")
REPO = os.path.dirname(PKG_DIR)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2,-Wall",
    "--expt-relaxed-constexpr",
    "-I" + os.path.join(REPO, "include"),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps() -> list[str]:
    out = [os.path.join(REPO, "include", f) for f in os.listdir(os.path.join(REPO, "include"))]
    out += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return out


def _stale(target: str, inputs: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(i) > t for i in inputs)


def _compile(src: str, extra: list[str], verbose_ptxas: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if _stale(obj, [src] + _deps()) or verbose_ptxas:
        cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose_ptxas:
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False, extra: list[str] | None = None) -> str:
    """Compile and link libqgmoe.so; returns its path.  Incremental by mtime."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    extra = list(extra or [])
    srcs = _sources()
    if force:
        for f in os.listdir(BUILD):
            if f.endswith(".o"):
                os.remove(os.path.join(BUILD, f))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, verbose_ptxas), srcs))
    if _stale(LIB, objs) or force:
        cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs,
               "-o", LIB, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


HOSTS_SRC = os.path.join(REPO, "tests", "c")
HOSTS_BUILD = os.path.join(HOSTS_SRC, "_build")


def build_host(name: str) -> str:
    """Compiles the plain-C host tests/c/<name>.c (a C99 program using only
    include/qgmoe.h and the CUDA runtime's C API) against the in-tree
    library; returns the executable's path.  Incremental by mtime."""
    src = os.path.join(HOSTS_SRC, name + ".c")
    exe = os.path.join(HOSTS_BUILD, name)
    lib = build()
    if _stale(exe, [src, lib, os.path.join(REPO, "include", "qgmoe.h")]):
        os.makedirs(HOSTS_BUILD, exist_ok=True)
        cuda = os.path.dirname(os.path.dirname(nvcc()))
        cmd = ["gcc", "-std=c99", "-O2", "-Wall", "-Wextra", "-pedantic", "-D_POSIX_C_SOURCE=200809L",
               "-I", os.path.join(REPO, "include"), "-I", os.path.join(cuda, "include"), src,
               "-o", exe, "-L", LIB_DIR, "-lqgmoe", "-L", os.path.join(cuda, "lib64"), "-lcudart",
               "-lm", "-Wl,-rpath," + LIB_DIR + ":" + os.path.join(cuda, "lib64")]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"gcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return exe


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
