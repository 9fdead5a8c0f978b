"""The C-ABI library loads without a GPU, exports every symbol that
include/fsa_sm100.h declares, and rejects bad arguments before touching CUDA."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from fusesampleagg_b200 import _lib

REPO = Path(__file__).resolve().parents[1]
HEADERS = sorted((REPO / "include").glob("*.h"))


def declared_symbols() -> set[str]:
    names = set()
    for h in HEADERS:
        text = h.read_text()
        names |= set(re.findall(r"FSA_API\s+[\w\s\*]+?\b(fsa_\w+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("fsa_sample_agg_forward", "fsa_sample_agg_backward",
                     "fsa_sample_agg_2hop_forward", "fsa_sample_agg_2hop_backward",
                     "fsa_fill_zero_f32"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_every_declared_symbol():
    assert declared_symbols() == set(_lib.SIGNATURES)


def test_header_compiles_as_c(tmp_path):
    import subprocess

    src = tmp_path / "t.c"
    src.write_text('#include "fsa_sm100.h"\nint main(void){return FSA_OK;}\n')
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{REPO / 'include'}", "-c",
                    str(src), "-o", str(tmp_path / "t.o")], check=True)


L = _lib.LIB
NULL = None


@pytest.mark.parametrize("fanout", [-1, 1025])
def test_forward_rejects_bad_fanout(fanout):
    assert L.fsa_sample_agg_forward(NULL, NULL, 10, 10, NULL, 4, NULL, 4, 0, fanout, 1,
                                    NULL, NULL, NULL, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT


def test_zero_sized_calls_are_noops_without_cuda():
    assert L.fsa_sample_agg_forward(NULL, NULL, 10, 10, NULL, 4, NULL, 0, 0, 3, 1,
                                    NULL, NULL, NULL, NULL) == _lib.FSA_OK
    assert L.fsa_sample_agg_forward(NULL, NULL, 10, 10, NULL, 4, NULL, 5, 0, 0, 1,
                                    NULL, NULL, NULL, NULL) == _lib.FSA_OK
    assert L.fsa_sample_agg_2hop_forward(NULL, NULL, 10, 10, NULL, 4, NULL, 5, 0, 0, 3, 1,
                                         NULL, NULL, NULL, NULL, 0, NULL, 0,
                                         NULL) == _lib.FSA_OK
    assert L.fsa_sample_agg_2hop_backward(NULL, NULL, NULL, 0, 4, 3, 2, NULL, 10,
                                          NULL) == _lib.FSA_OK
    assert L.fsa_fill_zero_f32(NULL, 0, NULL) == _lib.FSA_OK


@pytest.mark.parametrize("f1,f2", [(-1, 2), (2, -1), (12000, 1), (1000, 12)])
def test_2hop_rejects_bad_fanouts(f1, f2):
    assert L.fsa_sample_agg_2hop_forward(NULL, NULL, 10, 10, NULL, 4, NULL, 5, 0, f1, f2, 1,
                                         NULL, NULL, NULL, NULL, 0, NULL, 0,
                                         NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    assert L.fsa_sample_agg_2hop_backward(NULL, NULL, NULL, 5, 4, f1, f2, NULL, 10,
                                          NULL) == _lib.FSA_ERR_INVALID_ARGUMENT


def test_null_required_pointers_rejected():
    assert L.fsa_sample_agg_forward(NULL, NULL, 10, 10, NULL, 4, NULL, 5, 0, 3, 1,
                                    NULL, NULL, NULL, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    assert L.fsa_fill_zero_f32(NULL, 16, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    assert L.fsa_fill_zero_f32(NULL, -1, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT


def test_negative_sizes_rejected():
    assert L.fsa_sample_agg_forward(NULL, NULL, -1, 10, NULL, 4, NULL, 5, 0, 3, 1,
                                    NULL, NULL, NULL, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    assert L.fsa_sample_agg_forward(NULL, NULL, 10, 10, NULL, 4, NULL, 5, -3, 3, 1,
                                    NULL, NULL, NULL, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    assert L.fsa_sample_agg_backward(NULL, NULL, NULL, -1, 4, 3, NULL, 10,
                                     NULL) == _lib.FSA_ERR_INVALID_ARGUMENT


def test_workspace_size():
    assert L.fsa_sample_agg_2hop_workspace_size(0, 15, 10, 0, 0) == 0
    assert L.fsa_sample_agg_2hop_workspace_size(8, 0, 10, 0, 0) == 0
    with_ids = L.fsa_sample_agg_2hop_workspace_size(1024, 15, 10, 1, 1)
    without = L.fsa_sample_agg_2hop_workspace_size(1024, 15, 10, 0, 0)
    assert 0 < with_ids < without
    assert with_ids % 256 == 0 and without % 256 == 0
    # without requested ids the workspace also holds samples1 and samples2
    assert without - with_ids >= 4 * 1024 * 15 * 11


def test_2hop_forward_rejects_small_workspace():
    args = (1, 1, 10, 10, 1, 4, 1, 5, 0, 3, 2, 1, 1, NULL, NULL)
    need = L.fsa_sample_agg_2hop_workspace_size(5, 3, 2, 0, 0)
    assert L.fsa_sample_agg_2hop_forward(*args, 256, need - 1, NULL, 0,
                                         NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    assert L.fsa_sample_agg_2hop_forward(*args, 8, need, NULL, 0,
                                         NULL) == _lib.FSA_ERR_INVALID_ARGUMENT  # misaligned
    assert L.fsa_sample_agg_2hop_forward(*args, NULL, need, NULL, 0,
                                         NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    # a zero-fill request needs a buffer
    assert L.fsa_sample_agg_2hop_forward(*args, 256, need, NULL, 16,
                                         NULL) == _lib.FSA_ERR_INVALID_ARGUMENT


def test_status_strings():
    assert L.fsa_status_string(0) == b"ok"
    assert L.fsa_status_string(1) == b"invalid argument"
    assert L.fsa_status_string(2) == b"CUDA runtime error"
    assert L.fsa_status_string(99) == b"unknown status"


def test_check_raises_runtime_error():
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.check(_lib.FSA_ERR_INVALID_ARGUMENT, "x")
    _lib.check(_lib.FSA_OK, "x")


def test_phase_timing_without_calls_needs_no_cuda():
    _lib.phase_timing(True)
    times, calls = _lib.phase_times()
    _lib.phase_timing(False)
    assert calls == 0 and all(v == 0.0 for v in times.values())
    assert L.fsa_phase_times(None, None) == _lib.FSA_ERR_INVALID_ARGUMENT


def test_sharded_entry_points_reject_bad_tables_before_cuda():
    import ctypes as C

    two = (C.c_void_p * 2)(16, 32)
    nul = (C.c_void_p * 2)(16, None)
    # (table, shard_rows, num_shards, num_nodes): count, coverage, null, alignment
    bad = [(two, 5, 0, 10), (two, 5, _lib.MAX_SHARDS + 1, 10), (two, 4, 2, 10),
           (nul, 5, 2, 10), ((C.c_void_p * 2)(16, 36), 5, 2, 10), (two, 0, 2, 10)]
    for table, rows, n, nodes in bad:
        assert L.fsa_sample_agg_2hop_forward_sharded(
            NULL, NULL, nodes, 10, table, rows, n, 4, NULL, 5, 0, 3, 2, 1, NULL, NULL, NULL,
            NULL, 0, NULL, 0, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
        assert L.fsa_sample_agg_2hop_backward_sharded(
            NULL, NULL, NULL, 5, 4, 3, 2, table, rows, n, nodes,
            NULL) == _lib.FSA_ERR_INVALID_ARGUMENT


def test_ipc_and_peer_helpers_reject_null_arguments():
    assert L.fsa_ipc_export(NULL, NULL, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    assert L.fsa_ipc_open(NULL, 0, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    assert L.fsa_ipc_close(NULL, 0) == _lib.FSA_ERR_INVALID_ARGUMENT


# ---------------------------------------------------------------------------
# The torch binding (_fsa_torch): loads without a GPU, links this library
# ---------------------------------------------------------------------------

def test_torch_binding_loads_and_exposes_the_operator():
    from fusesampleagg_b200 import _fsa_torch

    for name in ("sample_agg", "sample_agg_with_samples", "sample_agg_2hop",
                 "sample_agg_2hop_with_samples"):
        assert callable(getattr(_fsa_torch, name))


def test_torch_binding_links_the_c_abi_library_from_its_own_directory():
    import subprocess

    from fusesampleagg_b200 import _fsa_torch

    out = subprocess.run(["readelf", "-d", _fsa_torch.__file__], check=True,
                         capture_output=True, text=True).stdout
    assert "[libfsa_sm100.so]" in out
    assert "$ORIGIN" in out


def test_torch_binding_rejects_cpu_tensors_before_cuda():
    import torch

    from fusesampleagg_b200 import _fsa_torch

    rp = torch.zeros(3, dtype=torch.int32)
    x = torch.zeros(2, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        _fsa_torch.sample_agg_2hop_with_samples(rp, rp, x, rp, 2, 2, 1, 0)
    with pytest.raises(RuntimeError, match="CUDA"):
        _fsa_torch.sample_agg_with_samples(rp, rp, x, rp, 2, 1, 0)


def test_exchange_bytes_layout():
    """Owner-computes sharded backward's region size: a 256-byte header,
    then per root 4 (f1 + f1 f2) bytes of ids and 4 D bytes of upstream
    gradient, each padded to 16 bytes."""
    assert L.fsa_exchange_bytes(0, 15, 10, 100) == 256
    assert L.fsa_exchange_bytes(1024, 15, 10, 100) == 256 + 1024 * (672 + 400)
    assert L.fsa_exchange_bytes(3, 2, 1, 3) == 256 + 3 * (16 + 16)
    assert L.fsa_exchange_bytes(-1, 15, 10, 100) == 0
    assert L.fsa_exchange_bytes(4, 5, 2400, 8) == 0  # over the 12000-entry limit


def test_exchange_entry_points_reject_bad_arguments_before_cuda():
    fake = 1 << 20  # aligned, never dereferenced: every call returns first
    assert L.fsa_sharded_publish_2hop(fake, 1024, fake, fake, fake, 64, 100, 15, 10,
                                      NULL) == _lib.FSA_ERR_INVALID_ARGUMENT  # region too small
    assert L.fsa_sharded_publish_2hop(fake + 8, 1 << 20, fake, fake, fake, 4, 100, 15, 10,
                                      NULL) == _lib.FSA_ERR_INVALID_ARGUMENT  # misaligned
    assert L.fsa_sharded_publish_2hop(fake, 1 << 20, NULL, fake, fake, 4, 100, 15, 10,
                                      NULL) == _lib.FSA_ERR_INVALID_ARGUMENT  # no gradient
    ptrs = (ctypes.c_void_p * 2)(fake, fake)
    pull = L.fsa_sample_agg_2hop_backward_sharded_pull
    assert pull(ptrs, 1 << 20, 2, 2, fake, 10, 20, 8, 3, 2, NULL, 0, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    assert pull(ptrs, 1 << 20, 2, 0, fake, 10, 21, 8, 3, 2, NULL, 0, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    assert pull(ptrs, 100, 2, 0, fake, 10, 20, 8, 3, 2, NULL, 0, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    bad = (ctypes.c_void_p * 2)(fake, None)
    assert pull(bad, 1 << 20, 2, 0, fake, 10, 20, 8, 3, 2, NULL, 0, NULL) == _lib.FSA_ERR_INVALID_ARGUMENT
    # nothing to add: returns before any CUDA call
    assert pull(ptrs, 1 << 20, 2, 0, fake, 10, 20, 8, 0, 2, NULL, 0, NULL) == _lib.FSA_OK
    # a touched-row list smaller than regions x records x f1 x f2
    assert pull(ptrs, 256 + 16 * (32 + 32), 2, 0, fake, 10, 20, 8, 3, 2, fake, 10,
                NULL) == _lib.FSA_ERR_INVALID_ARGUMENT

