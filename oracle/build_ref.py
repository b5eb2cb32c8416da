"""Build the reference's own IBCS/SIP CUDA kernels for sm_100a into oracle/_ref/.

ORACLE INFRASTRUCTURE (test-only). The reference (AB-Attention) ships its IBCS
and SIP kernels as CUDA sources (csrc/ibcs.cu, csrc/sip.cu) built with
`--use_fast_math` for sm_90a (setup.py:10-31). Their instructions (mma.sync,
ldmatrix, cp.async, CUB) are legal on sm_100a, so this recipe compiles the
sources where they lie in the reference checkout, together with the small
harness files beside this script, into `oracle/_ref/abx_ref*.so`. The shared
object travels to the GPU box and is the bit-exact oracle for every IBCS stage
and for SIP. The reference's own build system (setup.py) is not used.

Usage: python oracle/build_ref.py [--reference PATH]
"""
from __future__ import annotations

import argparse
import glob
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
DEFAULT_REFERENCE = Path("/root/reference")
SOURCES = ("ref_bindings.cpp", "ref_ibcs_harness.cu", "ref_sip_harness.cu")
# Same semantics as the reference build (setup.py:12-15), retargeted to sm_100a.
NVCC_FLAGS = [
    "-O3", "-gencode=arch=compute_100a,code=sm_100a",
    "--expt-extended-lambda", "--expt-relaxed-constexpr", "--use_fast_math",
]


def built_library() -> Path | None:
    hits = sorted(glob.glob(str(OUT / "abx_ref*.so")))
    return Path(hits[0]) if hits else None


def build(reference: Path = DEFAULT_REFERENCE, force: bool = False) -> Path | None:
    csrc = reference / "csrc"
    if not (csrc / "ibcs.cu").exists():
        return built_library()
    lib = built_library()
    inputs = [HERE / s for s in SOURCES] + [csrc / "ibcs.cu", csrc / "sip.cu"]
    if lib is not None and not force:
        newest = max(p.stat().st_mtime for p in inputs)
        if lib.stat().st_mtime >= newest:
            return lib
    OUT.mkdir(exist_ok=True)
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils import cpp_extension

    cpp_extension.load(
        name="abx_ref",
        sources=[str(HERE / s) for s in SOURCES],
        extra_include_paths=[str(csrc)],
        extra_cflags=["-O3"],
        extra_cuda_cflags=NVCC_FLAGS,
        build_directory=str(OUT),
        verbose=False,
    )
    # Keep only the shared object: ninja's bookkeeping lists every toolkit
    # header the build touched and is not needed to load the module.
    for leftover in (".ninja_deps", ".ninja_log", "build.ninja", *[p.name for p in OUT.glob("*.o")]):
        (OUT / leftover).unlink(missing_ok=True)
    return built_library()


def load():
    """Import the prebuilt reference module (works without the reference checkout)."""
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (the module links against libtorch)

    lib = built_library()
    if lib is None:
        raise RuntimeError("oracle/_ref is not built; run python oracle/build_ref.py")
    loader = importlib.machinery.ExtensionFileLoader("abx_ref", str(lib))
    spec = importlib.util.spec_from_file_location("abx_ref", str(lib), loader=loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    return module


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, default=DEFAULT_REFERENCE)
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    path = build(args.reference, args.force)
    print(path if path else "reference sources absent; nothing built")
    sys.exit(0 if path else 1)
