"""Builds libcmachine_b200.so in-tree: sm_100a CUDA kernels (nvcc) plus the C
session host (gcc), linked as one shared library with the C ABI of
include/gpu.h, include/qwen.h and include/qwen_b200.h.

    python -m cmachine_b200.build        (or __graft_entry__.build())
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
LIB = HERE / "libcmachine_b200.so"
CLI = HERE / "tcm-cuda"
BUILD = HERE / "_build"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall"]
CFLAGS = ["-O2", "-std=c11", "-fPIC", "-Wall", "-Wextra", "-D_GNU_SOURCE"]


def _sources():
    cu = sorted((HERE / "csrc").glob("*.cu"))
    c = sorted((HERE / "host").glob("*.c"))
    headers = sorted((HERE / "csrc").glob("*.cuh")) + sorted((HERE / "csrc").glob("*.h")) + sorted(
        (ROOT / "include").glob("*.h"))
    return cu, c, headers


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(" ".join(str(c) for c in cmd) + "\n" + proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")
    return proc


def build_library(verbose: bool = False) -> Path:
    cu, c, headers = _sources()
    BUILD.mkdir(exist_ok=True)
    objects = []
    for src in cu:
        obj = BUILD / (src.stem + ".cu.o")
        if _stale(obj, [src, *headers]):
            _run([NVCC, *NVFLAGS, "-c", str(src), "-o", str(obj)])
            if verbose:
                print("nvcc", src.name)
        objects.append(obj)
    for src in c:
        obj = BUILD / (src.stem + ".c.o")
        if _stale(obj, [src, *headers]):
            _run(["gcc", *CFLAGS, "-c", str(src), "-o", str(obj)])
            if verbose:
                print("gcc", src.name)
        objects.append(obj)
    if _stale(LIB, objects):
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-Xlinker", "-Bsymbolic", *map(str, objects), "-o", str(LIB),
              "-lpthread", "-ldl", "-lrt"])
        if verbose:
            print("link", LIB.name)
    # The serving executable (the reference's tcm-cuda; tcm-bounded-chat serves a ring).
    cli = HERE / "cli" / "tcm_cuda.c"
    if _stale(CLI, [cli, LIB]):
        _run(["gcc", "-O2", "-std=c11", "-Wall", str(cli), "-o", str(CLI), "-L", str(HERE), "-lcmachine_b200",
              "-Wl,-rpath,$ORIGIN"])
        if verbose:
            print("link", CLI.name)
    alias = HERE / "tcm-bounded-chat"
    if not alias.is_symlink():
        alias.symlink_to(CLI.name)
    return LIB


def build_oracle(verbose: bool = False) -> None:
    """The CPU checkers (test infrastructure): the oracle always, and the
    reference builds when the reference sources are present. The reference
    location is oracle/Makefile's REF, overridden by the CMACHINE_REFERENCE
    environment variable."""
    make = ["make", "-s", "-C", str(ROOT / "oracle")]
    ref = os.environ.get("CMACHINE_REFERENCE")
    if ref:
        make.append(f"REF={ref}")
    _run(make + ["liboracle.so"])
    _run(make + ["ref-if-present"])
    if verbose:
        print("oracle built")


if __name__ == "__main__":
    build_library(verbose=True)
    build_oracle(verbose=True)
