"""Builds the B200 backend: every source under csrc/ compiled by nvcc for
sm_100a into one shared library, defer_b200/libdefer_b200.so.

    python -m defer_b200.build            # incremental
    python -m defer_b200.build --clean

The host code (.cpp) is compiled by nvcc too so the whole library links
against one CUDA runtime (static cudart). Device code is compiled with
--fmad=false: every fused multiply-add in a kernel is an explicit fmaf,
and nothing else is contracted, so the arithmetic written in the source is
the arithmetic executed.
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
LIB = os.path.join(HERE, "libdefer_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-I", INCLUDE]
CU_FLAGS = ARCH + COMMON + ["-lineinfo", "--fmad=false", "-Xptxas", "-O3", "-diag-suppress", "550"]
CPP_FLAGS = ARCH + COMMON + ["-Xcompiler", "-O2"]


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def headers_mtime():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(INCLUDE, "defer_b200.h"))
    return max(os.path.getmtime(h) for h in hs)


def compile_one(src: str, force: bool, extra=()) -> str:
    s = os.path.join(CSRC, src)
    o = os.path.join(BUILD, src + ".o")
    if not force and os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), headers_mtime()):
        return o
    flags = CU_FLAGS if src.endswith(".cu") else CPP_FLAGS
    cmd = [NVCC] + flags + list(extra) + ["-x", "cu" if src.endswith(".cu") else "c++", "-c", s, "-o", o]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return o


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    a = ap.parse_args(argv)
    if a.clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    build(force=a.clean, verbose=True)


if __name__ == "__main__":
    main(sys.argv[1:])
