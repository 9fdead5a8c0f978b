"""ORACLE - test infrastructure, not product code.

numpy wrappers over oracle/libfsa_oracle.so, the sequential C restatement of
the reference operator (oracle/fsa_oracle.c).  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this module.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "libfsa_oracle.so"

_lib = None

_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_int = ctypes.c_int


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            from oracle.build import build_oracle

            build_oracle()
        L = ctypes.CDLL(str(LIB_PATH))
        L.fsa_oracle_sample_1hop.argtypes = [_i32p, _i32p, _i32p, _i64, _i64, _int, _u64,
                                             _i32p, _i32p, _int]
        L.fsa_oracle_sample_1hop.restype = None
        L.fsa_oracle_forward_1hop.argtypes = [_f32p, _i64, _i32p, _i32p, _i64, _int, _f32p, _int]
        L.fsa_oracle_forward_1hop.restype = None
        L.fsa_oracle_sample_2hop.argtypes = [_i32p, _i32p, _i32p, _i64, _i64, _int, _int, _u64,
                                             _i32p, _i32p, _int]
        L.fsa_oracle_sample_2hop.restype = None
        L.fsa_oracle_forward_2hop.argtypes = [_f32p, _i64, _i32p, _i64, _int, _int, _f32p, _int]
        L.fsa_oracle_forward_2hop.restype = None
        L.fsa_oracle_backward_1hop.argtypes = [_i32p, _i32p, _f32p, _i64, _i64, _int, _f32p]
        L.fsa_oracle_backward_1hop.restype = None
        L.fsa_oracle_backward_2hop.argtypes = [_f32p, _i32p, _i32p, _i64, _i64, _int, _int, _f32p]
        L.fsa_oracle_backward_2hop.restype = None
        L.fsa_oracle_xorshift_advance.argtypes = [_u64, _u64]
        L.fsa_oracle_xorshift_advance.restype = _u64
        L.fsa_oracle_row_state.argtypes = [_u64, _u64, _u64, _u64]
        L.fsa_oracle_row_state.restype = _u64
        L.fsa_oracle_bounded.argtypes = [_u64, ctypes.c_uint32]
        L.fsa_oracle_bounded.restype = ctypes.c_uint32
        _lib = L
    return _lib


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a), dtype=np.int32)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a), dtype=np.float32)


def sample_1hop(rowptr, col, frontier, fanout, seed, batch_offset=0, threads=1):
    rowptr, col, frontier = _i32(rowptr), _i32(col), _i32(frontier)
    B = frontier.shape[0]
    samples = np.full((B, fanout), -1, dtype=np.int32)
    takes = np.zeros(B, dtype=np.int32)
    if B and fanout:
        lib().fsa_oracle_sample_1hop(rowptr, col, frontier, B, batch_offset, fanout,
                                     seed, samples, takes, threads)
    return samples, takes


def forward_1hop(x, samples, takes, threads=1):
    x, samples, takes = _f32(x), _i32(samples), _i32(takes)
    B, fanout = samples.shape
    D = x.shape[1]
    out = np.zeros((B, D), dtype=np.float32)
    if B and fanout:
        lib().fsa_oracle_forward_1hop(x, D, samples, takes, B, fanout, out, threads)
    return out


def sample_2hop(rowptr, col, frontier, fanout1, fanout2, seed, batch_offset=0, threads=1):
    rowptr, col, frontier = _i32(rowptr), _i32(col), _i32(frontier)
    B = frontier.shape[0]
    s1 = np.full((B, fanout1), -1, dtype=np.int32)
    s2 = np.full((B, fanout1, fanout2), -1, dtype=np.int32)
    # fuseop/binding.cpp:183-185: no sampling at all when either fanout is 0.
    if B and fanout1 and fanout2:
        lib().fsa_oracle_sample_2hop(rowptr, col, frontier, B, batch_offset, fanout1, fanout2,
                                     seed, s1, s2, threads)
    return s1, s2


def forward_2hop(x, samples2, threads=1):
    x, samples2 = _f32(x), _i32(samples2)
    B, f1, f2 = samples2.shape
    D = x.shape[1]
    out = np.zeros((B, D), dtype=np.float32)
    if B and f1 and f2:
        lib().fsa_oracle_forward_2hop(x, D, samples2, B, f1, f2, out, threads)
    return out


def backward_1hop(samples, takes, grad_out, num_nodes):
    samples, takes, grad_out = _i32(samples), _i32(takes), _f32(grad_out)
    B, fanout = samples.shape
    D = grad_out.shape[1]
    grad_x = np.zeros((num_nodes, D), dtype=np.float32)
    if B and fanout:
        lib().fsa_oracle_backward_1hop(samples, takes, grad_out, B, D, fanout, grad_x)
    return grad_x


def backward_2hop(grad_out, samples1, samples2, num_nodes):
    grad_out, samples1, samples2 = _f32(grad_out), _i32(samples1), _i32(samples2)
    B, f1, f2 = samples2.shape
    D = grad_out.shape[1]
    grad_x = np.zeros((num_nodes, D), dtype=np.float32)
    if B and f1 and f2:
        lib().fsa_oracle_backward_2hop(grad_out, samples1, samples2, B, D, f1, f2, grad_x)
    return grad_x


def xorshift_advance(state: int, n: int) -> int:
    return int(lib().fsa_oracle_xorshift_advance(state, n))


def row_state(base: int, root: int, hop: int, pos: int) -> int:
    return int(lib().fsa_oracle_row_state(base, root, hop, pos))


def bounded(state: int, bound: int) -> int:
    return int(lib().fsa_oracle_bounded(state, bound))
