"""Drop-in acceptance: the reference's own test modules (tests/reference.py,
tests/test_correctness.py, tests/test_2hop.py), run unchanged against this
repository's ``fuseop`` package (fuseop/__init__.py at the repository root).

`python -m oracle.build --ref` copies the three files into
oracle/_ref/ref_tests (git-ignored, next to the reference op built from the
same checkout); they import ``from fuseop import ...``.  A child process
imports ``fuseop`` plainly from the repository root and checks that it got
this repository's package, not the reference op beside the copied tests
(pytest puts oracle/_ref on sys.path when it collects them).
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
REF_TESTS = REPO / "oracle" / "_ref" / "ref_tests"

BOOT = (
    "import sys, pathlib, fuseop; "
    "assert pathlib.Path(fuseop.__file__).resolve() == "
    "pathlib.Path(sys.argv[2]).resolve(), fuseop.__file__; "
    "import pytest; sys.exit(pytest.main(['-q', '-p', 'no:cacheprovider', sys.argv[1]]))"
)


def test_reference_test_modules_pass_against_this_package():
    if not (REF_TESTS / "test_correctness.py").exists():
        pytest.skip("reference tests not copied (python -m oracle.build --ref)")
    proc = subprocess.run([sys.executable, "-c", BOOT, str(REF_TESTS),
                           str(REPO / "fuseop" / "__init__.py")], cwd=REPO,
                          capture_output=True, text=True, timeout=600)
    tail = "\n".join(proc.stdout.splitlines()[-15:])
    assert proc.returncode == 0, tail
    summary = proc.stdout.strip().splitlines()[-1]
    assert " passed" in summary and "skipped" not in summary and "failed" not in summary, tail
