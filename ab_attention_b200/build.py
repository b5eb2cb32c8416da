"""Build libabx.so (the sm_100a kernels + C ABI) in-tree with nvcc.

The library is loaded by ab_attention_b200._lib through ctypes. Every kernel is
compiled for sm_100a only; the IBCS/SIP sources use --use_fast_math because
the reference kernels they must match bit-for-bit are built that way
(reference setup.py:12-15).

Usage: python -m ab_attention_b200.build [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libabx.so"
TORCH_LIB = PKG / "libabx_torch.so"  # torch.ops.ab_attention (csrc/torch_ops.cpp)
SOURCES = ("ibcs.cu", "sip.cu", "prefill.cu", "prefill_pair.cu", "capi.cu")
HEADERS = ("common.cuh", "ibcs.cuh", "tcgen05.cuh", "tma_host.cuh", "f32x2.cuh", "mix.cuh")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--use_fast_math", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-I", str(ROOT / "include"), "-I", str(CSRC),
    *ARCH,
]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else (shutil.which("nvcc") or "nvcc")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(force: bool = False, jobs: int = 4, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [ROOT / "include" / "abx.h"]
    objects = []
    commands = []
    for src in SOURCES:
        obj = BUILD / (Path(src).stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [CSRC / src, *headers]):
            commands.append([nvcc(), *NVCC_FLAGS, "-c", str(CSRC / src), "-o", str(obj)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
        return proc.stderr

    with futures.ThreadPoolExecutor(max_workers=max(1, jobs)) as pool:
        for out in pool.map(run, commands):
            if verbose and out:
                print(out)
    if force or commands or _stale(LIB, objects):
        # a SONAME, so the torch operator library records it and finds it beside itself
        run([nvcc(), "-shared", *ARCH, "-Xlinker", "-soname=libabx.so", "-o", str(LIB), *map(str, objects)])
    build_torch_ops(force, run)
    return LIB


def build_torch_ops(force: bool, run) -> Path:
    """libabx_torch.so: the TORCH_LIBRARY(ab_attention) operators over the C ABI,
    compiled against the installed torch and linked to libabx.so."""
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "torch_ops.cpp"
    if not (force or _stale(TORCH_LIB, [src, LIB, ROOT / "include" / "abx.h"])):
        return TORCH_LIB
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    includes = [f"-I{p}" for p in [str(ROOT / "include"), *cpp_extension.include_paths("cuda")]]
    libdirs = cpp_extension.library_paths("cuda")
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *includes, str(src), "-o", str(TORCH_LIB), f"-L{PKG}", "-l:libabx.so",
           *[f"-L{d}" for d in libdirs], "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10", "-lc10_cuda",
           "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{d}" for d in libdirs]]
    run(cmd)
    return TORCH_LIB


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=4)
    parser.add_argument("-v", "--verbose", action="store_true")
    args = parser.parse_args()
    print(build(args.force, args.jobs, args.verbose))
    sys.exit(0)
