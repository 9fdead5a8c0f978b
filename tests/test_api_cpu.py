"""Host-side behaviour of the public API without a GPU: the Python-side
error types and messages (fuseop/__init__.py:15-29), argument conversion,
the fanout and offset checks of the row-sharded entry, and the export list.
The C++ binding's RuntimeError checks (fuseop/binding.cpp:16-53, :119-135,
:200-218) are tested on the GPU through the public API
(tests/test_errors_gpu.py)."""

from __future__ import annotations

import pytest
import torch

import fusesampleagg_b200 as fsa


class FakeCuda:
    """Wraps a CPU tensor and reports itself as a CUDA tensor so the host
    checks can be exercised; no kernel is ever reached in these tests."""

    def __init__(self, t: torch.Tensor, device="cuda:0", contiguous=True):
        self.t = t
        self.is_cuda = True
        self.device = torch.device(device)
        self.dtype = t.dtype
        self._contig = contiguous

    def dim(self):
        return self.t.dim()

    def size(self, i=None):
        return self.t.size() if i is None else self.t.size(i)

    def numel(self):
        return self.t.numel()

    def is_contiguous(self):
        return self._contig

    @property
    def shape(self):
        return self.t.shape


def graph(**over):
    parts = dict(
        rowptr=FakeCuda(torch.tensor([0, 1, 2], dtype=torch.int32)),
        col=FakeCuda(torch.tensor([1, 0], dtype=torch.int32)),
        x=FakeCuda(torch.zeros(2, 4)),
        frontier=FakeCuda(torch.tensor([0, 1], dtype=torch.int32)),
    )
    parts.update(over)
    return parts


def test_public_names_match_reference():
    assert fsa.__all__ == [
        "fused_sample_agg",
        "fused_sample_agg_with_samples",
        "fused_sample_agg_2hop",
        "fused_sample_agg_2hop_with_samples",
    ]


@pytest.mark.parametrize("fn,args", [
    (fsa.fused_sample_agg, (2,)),
    (fsa.fused_sample_agg_with_samples, (2,)),
    (fsa.fused_sample_agg_2hop, (2, 2)),
    (fsa.fused_sample_agg_2hop_with_samples, (2, 2)),
])
def test_cpu_tensors_raise_value_error(fn, args):
    rowptr = torch.tensor([0, 1, 2], dtype=torch.int32)
    col = torch.tensor([1, 0], dtype=torch.int32)
    x = torch.zeros(2, 4)
    fr = torch.tensor([0], dtype=torch.int32)
    with pytest.raises(ValueError, match="must be CUDA tensors"):
        fn(rowptr, col, x, fr, *args)


@pytest.mark.parametrize("field,value,match", [
    ("rowptr", FakeCuda(torch.zeros(3, dtype=torch.int64)), "rowptr and col must have dtype"),
    ("col", FakeCuda(torch.zeros(2, dtype=torch.int64)), "rowptr and col must have dtype"),
    ("frontier", FakeCuda(torch.zeros(2, dtype=torch.int64)), "frontier must have dtype"),
    ("x", FakeCuda(torch.zeros(2, 4, dtype=torch.float64)), "x must have dtype"),
])
def test_python_dtype_checks_raise_type_error(field, value, match):
    g = graph(**{field: value})
    with pytest.raises(TypeError, match=match):
        fsa._check_python_inputs(g["rowptr"], g["col"], g["x"], g["frontier"])


@pytest.mark.parametrize("f1,f2,match", [
    (-1, 1, "non-negative"), (1, -1, "non-negative"),
    (2, 2**62, "too large"), (1000, 12, "too much shared memory"),
])
def test_fanout_2hop_limits(f1, f2, match):
    with pytest.raises(RuntimeError, match=match):
        fsa._check_fanout_2hop(f1, f2)
    fsa._check_fanout_2hop(1000, 11)
    fsa._check_fanout_2hop(0, 10**9)


@pytest.mark.parametrize("seed", [-1, 1 << 64])
def test_seed_outside_uint64_is_type_error(seed):
    with pytest.raises(TypeError):
        fsa._as_seed(seed)
    assert fsa._as_seed((1 << 64) - 1) == (1 << 64) - 1
    assert fsa._as_seed(3.7) == 3


def test_int64_conversion():
    with pytest.raises(TypeError):
        fsa._as_int64(1 << 63, "fanout")
    assert fsa._as_int64(True, "fanout") == 1


def test_batch_offset_must_be_non_negative():
    with pytest.raises(RuntimeError, match="batch_offset"):
        fsa._check_offset(-1)
    assert fsa._check_offset(5) == 5


def test_fuseop_package_serves_this_library():
    """`import fuseop` (the reference's package name, fuseop/__init__.py:209-214)
    gives the same four functions as fusesampleagg_b200."""
    import fuseop

    assert fuseop.__all__ == fsa.__all__
    for name in fuseop.__all__:
        assert getattr(fuseop, name) is getattr(fsa, name)


def test_bench_module_import_loads_no_library():
    """bench.py's reference arm must map only the reference's extension: the
    module itself imports neither this package nor its .so files."""
    import subprocess
    import sys

    code = ("import sys, bench; "
            "assert 'fusesampleagg_b200' not in sys.modules, 'package imported'; "
            "libs = bench.mapped_repo_libraries(); "
            "assert not libs, libs")
    proc = subprocess.run([sys.executable, "-c", code], cwd=str(fsa._lib.LIB_PATH.parents[1]),
                          capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]


def test_binding_raises_formatted_check_failures():
    """A TORCH_CHECK failure with a formatted message raised inside the C++
    binding comes back as RuntimeError, repeatedly (a binding built by a
    mismatched C++ toolchain crashed the process here instead)."""
    x = torch.zeros(4, 3)
    rp = torch.tensor([0, 0, 0, 0, 0], dtype=torch.int32)
    fr = torch.tensor([0], dtype=torch.int32)
    for _ in range(50):
        with pytest.raises(RuntimeError, match=r"grad_buffer shape must equal the features' "
                                               r"shape \(\[4, 2\] vs \[4, 3\]\)"):
            fsa._C.sample_agg_2hop_into(rp, rp[:0], x, fr, 2, 2, 1, 0, torch.zeros(4, 2), None)
