"""Builds libfsa_sm100.so in-tree with nvcc for sm_100a.

The library is a plain C-ABI shared object (include/fsa_sm100.h); it links
the CUDA runtime statically, so it loads into any process (including one
without a GPU, for symbol checks) and shares the device's primary context
with PyTorch.

Usage: ``python fusesampleagg_b200/build.py [--force] [--verbose]`` (run as a
script: importing the package loads the library this builds).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_NAME = "libfsa_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = [CSRC / "fsa_kernels.cu"]
DEPENDS = SOURCES + [CSRC / "fsa_rng.cuh", INCLUDE / "fsa_sm100.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def nvcc_command(output: Path, verbose_ptxas: bool = False) -> list[str]:
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-std=c++17",
        "-O3",
        "-lineinfo",
        "-shared",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        "-cudart",
        "static",
        f"-I{INCLUDE}",
        f"-I{CSRC}",
        "-DFSA_BUILD_SHARED",
        "-o",
        str(output),
        *[str(s) for s in SOURCES],
    ]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    return cmd


def is_stale(output: Path = LIB_PATH) -> bool:
    if not output.exists():
        return True
    mtime = output.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in DEPENDS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the library if it is missing or older than its sources."""
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = nvcc_command(tmp, verbose_ptxas=verbose)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(
            "nvcc failed building %s:\n%s\n%s" % (LIB_NAME, " ".join(cmd), proc.stderr)
        )
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = parser.parse_args()
    path = build(force=args.force, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    main()
