"""ctypes binding of libfsa_sm100.so (C ABI in include/fsa_sm100.h).

The library is required: importing this module raises ImportError when it is
missing or fails to load.  There is no CPU or eager fallback.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfsa_sm100.so"

FSA_OK = 0
FSA_ERR_INVALID_ARGUMENT = 1
FSA_ERR_CUDA = 2
FSA_ERR_SCRATCH_LIMIT = 3

FSA_STATUS_BAD_ROOT = 0x1
FSA_STATUS_BAD_ROW = 0x2
FSA_STATUS_BAD_NEIGHBOR = 0x4

MAX_FANOUT_1HOP = 1024
MAX_2HOP_ENTRIES = 12000
MAX_SHARDS = 64
IPC_HANDLE_BYTES = 64
NOALLOC_SCRATCH_BYTES = 4194304

# Every symbol include/fsa_sm100.h declares, with (restype, argtypes).
_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_u64 = ctypes.c_uint64
_int = ctypes.c_int

SIGNATURES = {
    "fsa_sample_agg_forward": (
        _int, [_p, _p, _i64, _i64, _p, _i64, _p, _i64, _i64, _i32, _u64, _p, _p, _p, _p]),
    "fsa_sample_agg_backward": (
        _int, [_p, _p, _p, _i64, _i64, _i32, _p, _i64, _p]),
    "fsa_sample_agg_2hop_workspace_size": (ctypes.c_size_t, [_i64, _i32, _i32, _int, _int]),
    "fsa_sample_agg_2hop_forward": (
        _int, [_p, _p, _i64, _i64, _p, _i64, _p, _i64, _i64, _i32, _i32, _u64, _p, _p, _p,
               _p, ctypes.c_size_t, _p, _i64, _p]),
    "fsa_sample_agg_2hop_forward_zero_rows": (
        _int, [_p, _p, _i64, _i64, _p, _i64, _p, _i64, _i64, _i32, _i32, _u64, _p, _p, _p,
               _p, ctypes.c_size_t, _p, _p, _i64, _p]),
    "fsa_sample_agg_2hop_forward_noalloc": (
        _int, [_p, _p, _i64, _i64, _p, _i64, _p, _i64, _i64, _i32, _i32, _u64, _p, _p, _p,
               _p, _i64, _p]),
    "fsa_sample_agg_2hop_forward_sharded": (
        _int, [_p, _p, _i64, _i64, ctypes.POINTER(_p), _i64, _i32, _i64, _p, _i64, _i64, _i32,
               _i32, _u64, _p, _p, _p, _p, ctypes.c_size_t, _p, _i64, _p]),
    "fsa_sample_agg_2hop_backward_sharded": (
        _int, [_p, _p, _p, _i64, _i64, _i32, _i32, ctypes.POINTER(_p), _i64, _i32, _i64, _p]),
    "fsa_sample_agg_2hop_backward": (
        _int, [_p, _p, _p, _i64, _i64, _i32, _i32, _p, _i64, _p]),
    "fsa_sample_agg_2hop_backward_sorted_workspace_size": (ctypes.c_size_t,
                                                            [_i64, _i64, _i32, _i32]),
    "fsa_sample_agg_2hop_backward_sorted": (
        _int, [_p, _p, _p, _i64, _i64, _i32, _i32, _p, _i64, _p, ctypes.c_size_t, _p]),
    "fsa_exchange_bytes": (ctypes.c_size_t, [_i64, _i32, _i32, _i64]),
    "fsa_sharded_publish_2hop": (_int, [_p, ctypes.c_size_t, _p, _p, _p, _i64, _i64, _i32, _i32,
                                        _p]),
    "fsa_sample_agg_2hop_backward_sharded_pull": (
        _int, [ctypes.POINTER(_p), ctypes.c_size_t, _i32, _i32, _p, _i64, _i64, _i64, _i32, _i32,
               _p, _i64, _p]),
    "fsa_sample_agg_2hop_forward_sharded_zero_rows": (
        _int, [_p, _p, _i64, _i64, ctypes.POINTER(_p), _i64, _i32, _i64, _p, _i64, _i64, _i32,
               _i32, _u64, _p, _p, _p, _p, ctypes.c_size_t, _p, _i64, _p, _i64, _p]),
    "fsa_fill_zero_f32": (_int, [_p, _i64, _p]),
    "fsa_zero_rows_f32": (_int, [_p, _i64, _i64, _p, _i64, _p]),
    "fsa_phase_timing": (_int, [_int]),
    "fsa_phase_times": (_int, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_i64)]),
    "fsa_ipc_export": (_int, [_p, _p, ctypes.POINTER(_u64)]),
    "fsa_ipc_open": (_int, [_p, _int, ctypes.POINTER(_p)]),
    "fsa_ipc_close": (_int, [_p, _int]),
    "fsa_enable_peer_access": (_int, [_int, _int]),
    "fsa_status_string": (ctypes.c_char_p, [_int]),
    "fsa_last_cuda_error": (_int, []),
    "fsa_launch_count": (_u64, []),
    "fsa_device_status": (_int, [_int, ctypes.POINTER(ctypes.c_uint32), _int]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is not built; run `python fusesampleagg_b200/build.py` "
            "(nvcc with sm_100a) before importing fusesampleagg_b200"
        )
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:
        raise ImportError(f"failed to load {LIB_PATH}: {exc}") from exc
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


LIB = _load()


def check(status: int, what: str) -> None:
    """Raises RuntimeError for a non-zero status of entry point `what`."""
    if status == FSA_OK:
        return
    text = LIB.fsa_status_string(status).decode()
    if status == FSA_ERR_CUDA:
        code = LIB.fsa_last_cuda_error()
        raise RuntimeError(f"{what} failed: {text} (cudaError {code})")
    raise RuntimeError(f"{what} failed: {text}")


def phase_timing(enable: bool) -> None:
    """Starts (clearing old records) or stops per-kernel event timing of
    the 2-hop forward."""
    check(LIB.fsa_phase_timing(int(bool(enable))), "fsa_phase_timing")


def phase_times() -> tuple[dict, int]:
    """Summed milliseconds of the recorded 2-hop forwards' plan, scan, draw
    and gather kernels, and the number of recorded calls."""
    ms = (ctypes.c_double * 4)()
    calls = _i64(0)
    check(LIB.fsa_phase_times(ms, ctypes.byref(calls)), "fsa_phase_times")
    return dict(zip(("plan", "scan", "draw", "gather"), list(ms))), int(calls.value)


def launch_count() -> int:
    """Kernels launched by the library so far in this process."""
    return int(LIB.fsa_launch_count())


def device_status(device: int, reset: bool = True) -> int:
    """Status word of `device` (FSA_STATUS_* bits); synchronises the device."""
    flags = ctypes.c_uint32(0)
    check(LIB.fsa_device_status(int(device), ctypes.byref(flags), int(bool(reset))),
          "fsa_device_status")
    return int(flags.value)
