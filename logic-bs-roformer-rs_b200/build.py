#!/usr/bin/env python3
"""Build the sm_100a engine library in-tree.

Compiles every ``csrc/*.cu`` (and the host-only ``csrc/*.cpp``) with nvcc for ``arch=compute_100a,code=sm_100a``
(``-lineinfo``, ``-O3``) and links ``lbrr/liblbrr_b200.so`` against cuFFT (the
only CUDA library the engine uses; no cuBLAS/cuBLASLt/cuDNN).  Objects go to
``_build/`` next to this file.  Incremental: a source is recompiled when it or
any header under ``csrc/`` or ``../include`` is newer than its object.

    python build.py [--verbose] [--ptxas-info]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIB = HERE / "lbrr" / "liblbrr_b200.so"
HOST = HERE / "host"
CLI = HERE / "lbrr" / "lbrr_b200"
CXX = os.environ.get("CXX", "g++")
CUDA_HOME = Path(NVCC_DIR := os.path.dirname(os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc"))).parent
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-I", str(CSRC), "-I", str(INCLUDE)]


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose: bool, ptxas_info: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()) and not ptxas_info:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0 or ptxas_info:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}")
    return obj


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, ptxas_info), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcufft", "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    build_cli(verbose)
    return LIB


def source_sha256() -> str:
    """SHA256 over the library, CLI and header sources (sorted by path), embedded
    in the CLI binary for its --bench identity record."""
    import hashlib
    h = hashlib.sha256()
    files = sorted(list(CSRC.glob("*")) + list(HOST.glob("*")) + list(INCLUDE.glob("*.h")))
    for f in files:
        if f.is_file():
            h.update(f.name.encode())
            h.update(f.read_bytes())
    return h.hexdigest()


def build_cli(verbose: bool = False) -> Path:
    """The host command-line front end (host/*.cpp), linked against the engine
    library it sits next to (rpath $ORIGIN) and the CUDA runtime."""
    srcs = sorted(HOST.glob("*.cpp"))
    deps = srcs + sorted(HOST.glob("*.h")) + [LIB, INCLUDE / "lbrr_gpu.h"]
    if CLI.exists() and CLI.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return CLI
    cmd = [CXX, "-O2", "-std=c++17", "-Wall", f'-DLBRR_SOURCE_SHA256="{source_sha256()}"',
           "-I", str(CUDA_HOME / "include"), *map(str, srcs), "-o", str(CLI),
           "-L", str(LIB.parent), "-llbrr_b200", "-L", str(CUDA_HOME / "lib64"), "-lcudart", "-lpthread",
           "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("host CLI build failed")
    return CLI


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_info))
