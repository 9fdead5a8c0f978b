"""Builds libfsa_sm100.so in-tree with nvcc for sm_100a, then the PyTorch
binding over it (_fsa_torch, g++ against the installed torch headers).

The library is a plain C-ABI shared object (include/fsa_sm100.h); it links
the CUDA runtime statically, so it loads into any process (including one
without a GPU, for symbol checks) and shares the device's primary context
with PyTorch.  The binding (csrc/fsa_torch.cpp) holds the operator's
autograd functions in C++ and finds the library next to itself ($ORIGIN).

Usage: ``python fusesampleagg_b200/build.py [--force] [--verbose]`` (run as a
script: importing the package loads the library this builds).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_NAME = "libfsa_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = [CSRC / "fsa_kernels.cu"]
DEPENDS = SOURCES + [CSRC / "fsa_rng.cuh", INCLUDE / "fsa_sm100.h"]

EXT_NAME = "_fsa_torch"
EXT_PATH = PKG_DIR / (EXT_NAME + sysconfig.get_config_var("EXT_SUFFIX"))
EXT_SOURCES = [CSRC / "fsa_torch.cpp"]
EXT_DEPENDS = EXT_SOURCES + [INCLUDE / "fsa_sm100.h", LIB_PATH]

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


def cxx_path() -> str:
    """The binding's C++ compiler: FSA_CXX, else the g++ on PATH.

    Not $CXX: the binding throws C++ exceptions (TORCH_CHECK) that unwind
    through libc10 / libtorch, so it must be built by the plain system
    toolchain those libraries were linked against.  A CXX wrapper that adds
    its own -B support-library directories produced a binding whose
    TORCH_CHECK failures with formatted messages crashed the process
    (SIGSEGV) instead of raising RuntimeError.
    """
    cxx = os.environ.get("FSA_CXX") or shutil.which("g++")
    if cxx is None:
        raise RuntimeError("g++ not found; set FSA_CXX")
    return cxx


def ext_command(output: Path) -> list[str]:
    """g++ line of the torch binding: torch's include and library paths and
    C++ ABI setting, linked to libfsa_sm100.so found beside it at run time."""
    import torch
    from torch.utils import cpp_extension

    abi = int(bool(torch._C._GLIBCXX_USE_CXX11_ABI))
    cmd = [
        cxx_path(),
        "-std=c++17",
        "-O2",
        "-shared",
        "-fPIC",
        "-fvisibility=hidden",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        f"-I{INCLUDE}",
        f"-I{sysconfig.get_paths()['include']}",
    ]
    cmd += [f"-I{p}" for p in cpp_extension.include_paths("cuda")]
    cmd += ["-o", str(output), *[str(s) for s in EXT_SOURCES]]
    cmd += [f"-L{p}" for p in cpp_extension.library_paths("cuda")]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
    cmd += [f"-L{PKG_DIR}", f"-l:{LIB_NAME}", "-Wl,-rpath,$ORIGIN"]
    return cmd


def is_stale(output: Path = LIB_PATH, depends=None) -> bool:
    if not output.exists():
        return True
    mtime = output.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in (DEPENDS if depends is None else depends))


def _run(cmd: list[str], what: str, tmp: Path, out: Path, verbose: bool) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("%s failed:\n%s\n%s" % (what, " ".join(cmd), proc.stderr))
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, out)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the library and then the torch binding, each if it is
    missing or older than its sources."""
    if force or is_stale():
        tmp = LIB_PATH.with_suffix(".so.tmp")
        _run(nvcc_command(tmp, verbose_ptxas=verbose), f"nvcc building {LIB_NAME}", tmp,
             LIB_PATH, verbose)
    if force or is_stale(EXT_PATH, EXT_DEPENDS):
        tmp = EXT_PATH.with_suffix(".tmp")
        _run(ext_command(tmp), f"g++ building {EXT_PATH.name}", tmp, EXT_PATH, verbose)
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
