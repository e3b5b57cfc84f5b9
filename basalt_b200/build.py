"""Builds libbasalt_cuda.so in-tree with nvcc for sm_100a.

The shared library links the CUDA runtime statically, so it only needs the driver at run time.
Object files go to ``_build/``; the library lands next to this file, where ``_lib.py`` loads it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIBRARY = PACKAGE / "libbasalt_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
          "-I", str(CSRC)]
SOURCES = ["kernels.cu", "gemm_tc.cu", "decode_fused.cu", "ops.cu", "ops_static.cu", "tensors.cu",
           "engine.cpp"]
HEADERS = ["kernels.h", "java_random.h", "epilogue.cuh", "device.cuh", "select.cuh"]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compiles the CUDA engine; returns the library path. Rebuilds only what changed."""
    BUILD.mkdir(exist_ok=True)
    compiler = nvcc()
    headers = [CSRC / h for h in HEADERS] + [INCLUDE / "basalt_cuda.h"]
    objects = []
    procs = []
    for src in SOURCES:
        path = CSRC / src
        obj = BUILD / (path.stem + ".o")
        objects.append(obj)
        if _newer(obj, [path, *headers]):
            lang = [] if src.endswith(".cu") else ["-x", "cu"]
            cmd = [compiler, *ARCH, *COMMON, *lang, "-c", str(path), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd))
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                                stderr=subprocess.STDOUT, text=True)))
    for src, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{out}")
        if verbose and out.strip():
            print(out)
    if _newer(LIBRARY, objects):
        cmd = [compiler, *ARCH, "-shared", "-cudart", "static", "-o", str(LIBRARY),
               *map(str, objects), "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd))
        result = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"linking libbasalt_cuda.so failed:\n{result.stdout}")
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose=True))
