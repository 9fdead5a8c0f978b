"""ORACLE build recipe - test infrastructure, not product code.

Builds two checkers:

* ``oracle/libfsa_oracle.so`` - the C restatement (oracle/fsa_oracle.c),
  gcc -O2 without fast-math (IEEE float order is part of parity).
* ``oracle/_ref/fuseop/`` - the reference operator itself, compiled from its
  own sources where they lie in the reference checkout
  (fuseop/binding.cpp + fuseop/fused_sample_agg.cu) with the flags of its
  setup.py (fuseop/setup.py:20-23: -O3 -std=c++17) for sm_100
  (TORCH_CUDA_ARCH_LIST=10.0, as a PyTorch build for B200 would choose), plus
  its Python package file so ``import fuseop`` gives the reference's own
  public API.  This does not run the reference's build system.  The output
  is git-ignored but travels to the GPU box with the working tree; it is
  where the bit-exact golden vectors (tests/golden/) come from and what
  ``bench.py --impl reference`` times.

Usage: ``python -m oracle.build [--ref --reference-root PATH]``; the
reference checkout may also be named by the FSA_REFERENCE_ROOT environment
variable.  There is no default location.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
REF_OUT = ORACLE_DIR / "_ref"
REF_PKG = REF_OUT / "fuseop"
REFERENCE_ROOT_ENV = "FSA_REFERENCE_ROOT"


def reference_root_from_env() -> Path | None:
    """The reference checkout named by FSA_REFERENCE_ROOT, if any."""
    v = os.environ.get(REFERENCE_ROOT_ENV)
    return Path(v) if v else None


def build_oracle(force: bool = False) -> Path:
    out = ORACLE_DIR / "libfsa_oracle.so"
    src = ORACLE_DIR / "fsa_oracle.c"
    if not force and out.exists() and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    tmp = out.with_suffix(".so.tmp")
    cmd = ["gcc", "-O2", "-std=c11", "-fopenmp", "-fPIC", "-shared", "-fvisibility=hidden",
           "-o", str(tmp), str(src)]
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


def reference_available(reference_root: Path | None) -> bool:
    return reference_root is not None and (reference_root / "fuseop" / "fused_sample_agg.cu").exists()


def ref_built() -> bool:
    return any(REF_PKG.glob("_C*.so")) and (REF_PKG / "__init__.py").exists()


def build_ref(reference_root: Path | None, force: bool = False) -> Path | None:
    """Compiles the reference op into oracle/_ref/fuseop (None if absent)."""
    if not reference_available(reference_root):
        return None
    if ref_built() and not force:
        return REF_PKG
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0"
    # torch's extension builder takes the host compiler from CXX; use the
    # system g++ (a CXX wrapper with its own support-library paths built
    # extensions whose formatted TORCH_CHECK failures crashed).
    gxx = shutil.which("g++")
    if gxx:
        os.environ["CXX"] = gxx
    from torch.utils.cpp_extension import load

    build_dir = REF_OUT / "build"
    build_dir.mkdir(parents=True, exist_ok=True)
    REF_PKG.mkdir(parents=True, exist_ok=True)
    src = reference_root / "fuseop"
    load(
        name="_C",
        sources=[str(src / "binding.cpp"), str(src / "fused_sample_agg.cu")],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=["-O3", "-std=c++17"],
        build_directory=str(build_dir),
        verbose=False,
    )
    built = build_dir / "_C.so"
    shutil.copyfile(built, REF_PKG / "_C.so")
    shutil.copyfile(src / "__init__.py", REF_PKG / "__init__.py")
    # The reference's pure-PyTorch aggregation helpers (tests/reference.py).
    ref_tests = REF_OUT / "ref_tests"
    ref_tests.mkdir(exist_ok=True)
    for name in ("reference.py", "test_correctness.py", "test_2hop.py", "__init__.py"):
        path = reference_root / "tests" / name
        if path.exists():
            shutil.copyfile(path, ref_tests / name)
    return REF_PKG


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--ref", action="store_true", help="also build the reference op")
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--reference-root", type=Path, default=reference_root_from_env(),
                        help=f"reference checkout (default: ${REFERENCE_ROOT_ENV})")
    args = parser.parse_args()
    print(build_oracle(force=args.force))
    if args.ref:
        if args.reference_root is None:
            parser.error(f"--ref needs --reference-root or ${REFERENCE_ROOT_ENV}")
        print(build_ref(args.reference_root, force=args.force))


if __name__ == "__main__":
    main()
