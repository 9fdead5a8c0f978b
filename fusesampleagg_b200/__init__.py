"""B200-native fused reservoir-sample + mean-aggregate operator for PyTorch.

Drop-in for the FuseSampleAgg Python API (fuseop/__init__.py:75-214): the
same four functions with the same arguments, return containers, autograd
saved-index replay and error types.  The autograd functions and output
allocation live in a C++ torch binding (_fsa_torch, csrc/fsa_torch.cpp)
that calls the C ABI of libfsa_sm100.so (include/fsa_sm100.h), which
launches hand-written sm_100a kernels on the caller's current CUDA stream.
There is no CPU fallback: the import fails when either is missing.

Sampled neighbour ids are bit-identical to the reference for the same
(graph, frontier, fanouts, replay_seed); forward outputs are bit-identical
as well (same fp32 summation order); feature gradients match to fp32
rounding (atomic accumulation order differs, as in the reference).

Two additions over the reference API, both keyword-only:

* ``batch_offset`` (default 0) is added to the batch index in the first-hop
  seeds, so a contiguous slice of a larger batch -- e.g. one GPU's share of
  the roots -- draws exactly the samples the whole batch would;
* ``grad_buffer`` (default None) takes a ``PersistentGradient``: the
  backward adds into that buffer instead of returning a fresh dense N x D
  gradient, and the buffer is cleared row by row (see PersistentGradient).
"""

from __future__ import annotations

import torch

from . import _lib

try:
    from . import _fsa_torch as _C
except ImportError as exc:  # no fallback: the binding is part of the build
    raise ImportError(
        "fusesampleagg_b200._fsa_torch is not built; run `python fusesampleagg_b200/build.py` "
        f"before importing fusesampleagg_b200 ({exc})") from exc

__all__ = [
    "fused_sample_agg",
    "fused_sample_agg_with_samples",
    "fused_sample_agg_2hop",
    "fused_sample_agg_2hop_with_samples",
]

_L = _lib.LIB
_U64 = 1 << 64
_I64_MIN = -(1 << 63)
_I64_MAX = (1 << 63) - 1


# ---------------------------------------------------------------------------
# Argument checks.  The Python-side ValueError / TypeError checks of
# fuseop/__init__.py:15-29 run here; the RuntimeError checks of
# fuseop/binding.cpp:16-53, :119-135 and :200-218 run in the C++ binding
# (csrc/fsa_torch.cpp).  The row-sharded entry (sharding.py), which calls the
# C ABI directly, uses the integer, fanout and offset checks below.
# ---------------------------------------------------------------------------

def _check_python_inputs(rowptr, col, x, frontier) -> None:
    if not all(t.is_cuda for t in (rowptr, col, x, frontier)):
        raise ValueError("rowptr, col, x, and frontier must be CUDA tensors")
    if rowptr.dtype != torch.int32 or col.dtype != torch.int32:
        raise TypeError("rowptr and col must have dtype torch.int32")
    if frontier.dtype != torch.int32:
        raise TypeError("frontier must have dtype torch.int32")
    if x.dtype != torch.float32:
        raise TypeError("x must have dtype torch.float32")


def _as_int64(value, what: str) -> int:
    v = int(value)
    if not _I64_MIN <= v <= _I64_MAX:
        raise TypeError(f"{what} does not fit a 64-bit signed integer")
    return v


def _as_seed(value) -> int:
    v = int(value)
    if not 0 <= v < _U64:
        raise TypeError("replay_seed must be an integer in [0, 2**64)")
    return v


def _check_fanout_2hop(fanout1: int, fanout2: int) -> None:
    if fanout1 < 0 or fanout2 < 0:
        raise RuntimeError("fanouts must be non-negative")
    if fanout1 != 0 and fanout2 > (_I64_MAX - fanout1) // fanout1:
        raise RuntimeError("fanout pair is too large")
    if fanout1 + fanout1 * fanout2 > _lib.MAX_2HOP_ENTRIES:
        raise RuntimeError("fanout pair requires too much shared memory; reduce fanout1 or fanout2")


def _check_offset(batch_offset) -> int:
    off = _as_int64(batch_offset, "batch_offset")
    if off < 0:
        raise RuntimeError("batch_offset must be non-negative")
    return off


class _DeviceGuard:
    """Makes `device` current for the duration of a call (like CUDAGuard)."""

    __slots__ = ("index", "prev")

    def __init__(self, device: torch.device):
        self.index = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = -1

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.index:
            self.prev = cur
            torch.cuda.set_device(self.index)
        return self

    def __exit__(self, *exc):
        if self.prev >= 0:
            torch.cuda.set_device(self.prev)
        return False


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_handle(device: torch.device) -> int:
    """cudaStream_t of the current stream of `device` (the raw-handle query
    when this torch build has it: a fraction of the cost of building a
    torch.cuda.Stream object on every call)."""
    if _raw_stream is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return _raw_stream(idx)
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t):
    return t.data_ptr() if t is not None else None


# ---------------------------------------------------------------------------
# Public API (fuseop/__init__.py:75-206)
# ---------------------------------------------------------------------------

def fused_sample_agg(rowptr, col, x, frontier, fanout, replay_seed=1234, save_indices=False,
                     *, batch_offset=0, grad_buffer=None, clear_grad_buffer=False):
    """Return the sampled 1-hop neighbor mean for each frontier node."""
    _check_python_inputs(rowptr, col, x, frontier)
    fanout = _as_int64(fanout, "fanout")
    seed = _as_seed(replay_seed)
    offset = _as_int64(batch_offset, "batch_offset")
    if clear_grad_buffer and grad_buffer is None:
        raise ValueError("clear_grad_buffer needs a grad_buffer")
    if grad_buffer is not None:
        buf = _buffer_tensor(grad_buffer)
        if clear_grad_buffer:
            grad_buffer.zero_()
        out, ids, flag = _C.sample_agg_into(rowptr, col, x, frontier, fanout, seed, offset, buf)
        grad_buffer._record(ids, flag)
        return out
    return _C.sample_agg(rowptr, col, x, frontier, fanout, seed, bool(save_indices), offset)


def fused_sample_agg_with_samples(rowptr, col, x, frontier, fanout, replay_seed=1234,
                                  *, batch_offset=0):
    """Return 1-hop means, sampled neighbor IDs, and valid sample counts.

    Returns a list ``[out[B,D], samples[B,fanout] (-1 padded), takes[B]]``;
    no autograd.
    """
    _check_python_inputs(rowptr, col, x, frontier)
    return _C.sample_agg_with_samples(rowptr, col, x, frontier, _as_int64(fanout, "fanout"),
                                      _as_seed(replay_seed),
                                      _as_int64(batch_offset, "batch_offset"))


def fused_sample_agg_2hop(rowptr, col, x, frontier, fanout1, fanout2, replay_seed=1234,
                          save_indices=False, *, batch_offset=0, grad_buffer=None,
                          clear_grad_buffer=False):
    """Return the nested sampled 2-hop neighbor mean for each frontier node.

    ``clear_grad_buffer=True`` (with a ``grad_buffer``) does what
    ``grad_buffer.zero_()`` right before the call would, inside the call:
    the rows are zeroed by the sampling kernel, whose draws leave the memory
    system idle, instead of by a kernel of their own.
    """
    _check_python_inputs(rowptr, col, x, frontier)
    f1 = _as_int64(fanout1, "fanout1")
    f2 = _as_int64(fanout2, "fanout2")
    seed = _as_seed(replay_seed)
    offset = _as_int64(batch_offset, "batch_offset")
    if clear_grad_buffer and grad_buffer is None:
        raise ValueError("clear_grad_buffer needs a grad_buffer")
    if grad_buffer is not None:
        buf = _buffer_tensor(grad_buffer)
        rows = grad_buffer._rows_to_clear() if clear_grad_buffer else None
        out, ids, flag = _C.sample_agg_2hop_into(rowptr, col, x, frontier, f1, f2, seed, offset,
                                                 buf, rows)
        if clear_grad_buffer:
            grad_buffer._cleared()
        grad_buffer._record(ids, flag)
        return out
    return _C.sample_agg_2hop(rowptr, col, x, frontier, f1, f2, seed, bool(save_indices),
                              offset)


def fused_sample_agg_2hop_with_samples(rowptr, col, x, frontier, fanout1, fanout2,
                                       replay_seed=1234, *, batch_offset=0):
    """Return nested means and sampled first- and second-hop neighbor IDs.

    Returns a tuple ``(out[B,D], samples1[B,f1], samples2[B,f1,f2])``; no
    autograd.
    """
    _check_python_inputs(rowptr, col, x, frontier)
    return _C.sample_agg_2hop_with_samples(rowptr, col, x, frontier,
                                           _as_int64(fanout1, "fanout1"),
                                           _as_int64(fanout2, "fanout2"), _as_seed(replay_seed),
                                           _as_int64(batch_offset, "batch_offset"))


# ---------------------------------------------------------------------------
# Persistent gradient buffer (opt-in; no counterpart in the reference)
# ---------------------------------------------------------------------------

class PersistentGradient:
    """A feature-table gradient kept across steps and cleared row by row.

    The reference's backward hands autograd a fresh dense N x D gradient on
    every call (at::zeros, fuseop/binding.cpp:137, :220): 4 N D bytes of
    zero fill per step although a step touches only the sampled rows.
    Passing ``grad_buffer=buf`` to ``fused_sample_agg`` or
    ``fused_sample_agg_2hop`` makes the backward add into ``buf.grad``
    instead, and autograd then produces no gradient for ``x`` from that call.
    ``buf.zero_()`` clears the rows that the calls since the previous
    ``zero_()`` sample -- their saved ids -- rather than the whole table.

    ``buf.grad`` is one tensor for the buffer's lifetime.  To train through
    an optimizer, alias it once (``x.grad = buf.grad``) and call
    ``buf.zero_()`` where ``optimizer.zero_grad()`` would go (never
    ``zero_grad(set_to_none=True)``, which drops the alias).  Calls are
    stream-ordered on the current stream like the rest of the API.

    Rows of a forward whose backward has not run yet are cleared again by
    every later ``zero_()`` until that backward has run (or its graph has
    been freed), so ``zero_()`` may sit anywhere between steps.
    """

    def __init__(self, x: torch.Tensor):
        if not (x.is_cuda and x.dim() == 2):
            raise ValueError("PersistentGradient needs the 2-D CUDA feature tensor")
        with _DeviceGuard(x.device):
            self.grad = torch.empty(tuple(x.shape), dtype=torch.float32, device=x.device)
            _lib.check(_L.fsa_fill_zero_f32(self.grad.data_ptr(), self.grad.numel(),
                                            _stream_handle(x.device)), "fsa_fill_zero_f32")
        self._touched: list[tuple[torch.Tensor, torch.Tensor]] = []

    def _record(self, ids, flag) -> None:
        if ids is not None:
            self._touched.append((ids, flag))

    @property
    def pending_rows(self) -> int:
        """Saved-id entries (rows, with repeats and -1 padding) that the next
        ``zero_()`` will clear."""
        return sum(int(ids.numel()) for ids, _ in self._touched)

    def zero_(self) -> "PersistentGradient":
        """Zeroes the rows touched since the last call (one fsa_zero_rows_f32
        launch over the recorded calls' saved ids)."""
        rows = self._rows_to_clear()
        if rows is not None:
            _C.zero_rows(self.grad, rows)
        self._cleared()
        return self

    def _rows_to_clear(self):
        """The recorded calls' saved ids as one int32 list, or None."""
        if not self._touched:
            return None
        if len(self._touched) == 1:
            return self._touched[0][0].reshape(-1)
        return torch.cat([ids.reshape(-1) for ids, _ in self._touched])

    def _cleared(self) -> None:
        """Forgets the recorded calls whose rows were just zeroed, except
        those still awaiting their backward (their rows will be touched
        again): still pending, and their graph -- which holds the other
        reference to the flag -- is alive."""
        self._touched = [(ids, flag) for ids, flag in self._touched
                         if int(flag[0]) != 0 and flag._use_count() > 1]


def _buffer_tensor(buf) -> torch.Tensor:
    if not isinstance(buf, PersistentGradient):
        raise TypeError("grad_buffer must be a fusesampleagg_b200.PersistentGradient")
    return buf.grad


def launch_count() -> int:
    """Kernels launched by libfsa_sm100.so in this process."""
    return _lib.launch_count()


def device_status(device=None, reset: bool = True) -> int:
    """OR of FSA_STATUS_* bits raised by kernels on `device` since the last
    reset (out-of-range root / row / neighbour ids).  Synchronises."""
    if device is None:
        device = torch.cuda.current_device()
    elif isinstance(device, torch.device):
        device = device.index if device.index is not None else torch.cuda.current_device()
    return _lib.device_status(int(device), reset)
