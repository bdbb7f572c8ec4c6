"""Builds the sm_100a shared library ``lib/libgns_b200.so`` in-tree with nvcc.

Usage: ``python -m gram_newton_schulz_ampere_b200.build [--force] [--verbose]``.
The library links the CUDA runtime statically and resolves the driver entry
point it needs (``cuTensorMapEncodeTiled``) at run time, so it loads on a host
without a GPU driver and is self-contained on the GPU box.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC_DIR = PACKAGE_DIR / "csrc"
LIB_DIR = PACKAGE_DIR / "lib"
LIB_PATH = LIB_DIR / "libgns_b200.so"
INCLUDE_DIR = PACKAGE_DIR.parent / "include"

SOURCES = ("gemm_launch.cu", "ns_chain.cu", "optim_kernels.cu", "small_chain.cu")
ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")
NVCC_FLAGS = (
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
)


def nvcc_path() -> str:
    candidates = [
        shutil.which("nvcc"),
        os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"),
    ]
    for candidate in candidates:
        if candidate and os.path.exists(candidate):
            return candidate
    raise RuntimeError("nvcc not found; set CUDA_HOME")


def _inputs() -> list[Path]:
    files = [CSRC_DIR / name for name in SOURCES]
    files += sorted(CSRC_DIR.glob("*.cuh")) + sorted(CSRC_DIR.glob("*.h"))
    files += sorted(INCLUDE_DIR.glob("*.h"))
    return files


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(path.stat().st_mtime > built for path in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compiles every source into one shared library; returns its path."""
    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    nvcc = nvcc_path()
    obj_dir = PACKAGE_DIR / "_build"
    obj_dir.mkdir(exist_ok=True)
    objects = []
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    for name in SOURCES:
        src = CSRC_DIR / name
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", str(INCLUDE_DIR), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *objects]
    if verbose:
        print(" ".join(link), flush=True)
    subprocess.run(link, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-verbose", action="store_true")
    args = parser.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
