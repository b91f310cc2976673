"""Build the native parts of gpuos_b200 in-tree for sm_100a.

    python -m gpuos_b200._build          # incremental
    python -m gpuos_b200._build --force  # rebuild everything

Outputs (next to this file, git-ignored, shipped with the tree):
    libgpuos_b200.so   the executor (CUDA kernels + C++ runtime + C ABI),
                       cudart linked statically
    gpuos_ext*.so      the Python module with the reference's API

No GPU is needed to build: nvcc cross-compiles for sm_100a.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
ROOT = HERE.parent
BUILD = ROOT / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB = HERE / "libgpuos_b200.so"
EXT = HERE / ("gpuos_ext" + sysconfig.get_config_var("EXT_SUFFIX"))

DEV_HEADERS = [CSRC / "gpuos_abi.h", CSRC / "ops.cuh", CSRC / "executor.cuh", CSRC / "batch.cuh"]
HOST_HEADERS = [CSRC / "gpuos_abi.h", CSRC / "runtime.h", ROOT / "include" / "gpuos_b200.h"]


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    r = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... -> exit {r.returncode}")
    return r


def build_lib(force=False, verbose=False) -> Path:
    BUILD.mkdir(exist_ok=True)
    kobj = BUILD / "kernels.o"
    robj = BUILD / "runtime.o"
    if force or _stale(kobj, [CSRC / "kernels.cu", *DEV_HEADERS]):
        _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
              "-c", CSRC / "kernels.cu", "-o", kobj], verbose)
    nobj = BUILD / "noalloc.o"
    if force or _stale(nobj, [CSRC / "noalloc.cu", ROOT / "include" / "gpuos_b200.h", *DEV_HEADERS]):
        _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
              "-c", CSRC / "noalloc.cu", "-o", nobj], verbose)
    if force or _stale(robj, [CSRC / "runtime.cpp", *HOST_HEADERS]):
        _run(["g++", "-std=c++17", "-O2", "-fPIC", "-Wall", "-Wno-unused-parameter",
              f"-I{CUDA_HOME / 'include'}", "-c", CSRC / "runtime.cpp", "-o", robj], verbose)
    if force or _stale(LIB, [kobj, robj, nobj]):
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, kobj, robj, nobj,
              "-Xlinker", "--no-undefined", "-lpthread", "-ldl", "-lrt"], verbose)
    return LIB


def build_ext(force=False, verbose=False) -> Path:
    import torch
    from torch.utils import cpp_extension

    lib = build_lib(force, verbose)
    if not (force or _stale(EXT, [CSRC / "ext.cpp", lib, *HOST_HEADERS])):
        return EXT
    inc = [f"-I{p}" for p in cpp_extension.include_paths()]
    inc += [f"-I{sysconfig.get_paths()['include']}", f"-I{CUDA_HOME / 'include'}"]
    tlib = cpp_extension.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
          "-DTORCH_EXTENSION_NAME=gpuos_ext", *inc, CSRC / "ext.cpp", "-o", EXT,
          f"-L{HERE}", "-lgpuos_b200", f"-L{tlib}", "-ltorch_python", "-ltorch", "-ltorch_cpu",
          "-lc10", "-lc10_cuda", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{tlib}"], verbose)
    return EXT


def build(force=False, verbose=False):
    build_ext(force, verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
    print(EXT)
