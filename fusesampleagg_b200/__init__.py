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

One addition over the reference API: a keyword-only ``batch_offset``
(default 0) that is added to the batch index in the first-hop seeds, so a
contiguous slice of a larger batch -- e.g. one GPU's share of the roots --
draws exactly the samples the whole batch would.
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
# Argument checks (fuseop/__init__.py:15-29 and fuseop/binding.cpp:16-53)
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


def _check_graph_inputs(rowptr, col, x, frontier) -> None:
    dev = x.device
    if not (x.is_cuda and rowptr.is_cuda and col.is_cuda and frontier.is_cuda):
        raise RuntimeError("all inputs must be CUDA tensors")
    if rowptr.device != dev or col.device != dev or frontier.device != dev:
        raise RuntimeError("all inputs must be on the same CUDA device")
    i32 = torch.int32
    if rowptr.dtype != i32 or col.dtype != i32 or frontier.dtype != i32:
        raise RuntimeError("rowptr, col, and frontier must be int32")
    if x.dtype != torch.float32:
        raise RuntimeError("x must be float32")
    if rowptr.dim() != 1 or col.dim() != 1 or x.dim() != 2 or frontier.dim() != 1:
        raise RuntimeError("expected rowptr[N+1], col[E], x[N,D], and frontier[B]")
    if not (x.is_contiguous() and rowptr.is_contiguous() and col.is_contiguous()
            and frontier.is_contiguous()):
        raise RuntimeError("all inputs must be contiguous")
    if rowptr.numel() != x.size(0) + 1:
        raise RuntimeError("rowptr length must equal N+1")


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


def _check_fanout_1hop(fanout: int) -> None:
    if fanout < 0:
        raise RuntimeError("fanout must be non-negative")
    if fanout > _lib.MAX_FANOUT_1HOP:
        raise RuntimeError(f"fanout exceeds the supported maximum of {_lib.MAX_FANOUT_1HOP}")


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


def _zeroed(num_nodes: int, dim: int, device: torch.device, stream: int) -> torch.Tensor:
    grad = torch.empty((num_nodes, dim), dtype=torch.float32, device=device)
    _lib.check(_L.fsa_fill_zero_f32(grad.data_ptr(), grad.numel(), stream), "fsa_fill_zero_f32")
    return grad


def _grad_buffer(zeroed, num_nodes, dim, device, stream) -> torch.Tensor:
    """The dense gradient: the buffer the forward already zeroed, else a new
    zero-filled one (the reference's at::zeros, fuseop/binding.cpp:137, :220)."""
    if zeroed is not None and tuple(zeroed.shape) == (num_nodes, dim) and zeroed.device == device:
        return zeroed
    return _zeroed(num_nodes, dim, device, stream)


# ---------------------------------------------------------------------------
# Backward launch wrappers over ctypes (fuseop/binding.cpp:119-145, :200-231):
# the public functions' autograd runs in the C++ binding; these serve direct
# replays of saved ids.
# ---------------------------------------------------------------------------

def _backward_1hop(samples, takes, grad_out, num_nodes):
    if not (samples.is_cuda and takes.is_cuda and grad_out.is_cuda):
        raise RuntimeError("backward inputs must be CUDA tensors")
    if samples.dtype != torch.int32 or takes.dtype != torch.int32:
        raise RuntimeError("samples and takes must be int32")
    if not (samples.device == takes.device == grad_out.device):
        raise RuntimeError("backward inputs must be on the same CUDA device")
    if grad_out.dtype != torch.float32 or grad_out.dim() != 2:
        raise RuntimeError("grad_out must be a float32 matrix")
    if (samples.dim() != 2 or takes.dim() != 1 or samples.size(0) != grad_out.size(0)
            or takes.size(0) != grad_out.size(0)):
        raise RuntimeError("saved sample shapes do not match grad_out")
    if not (samples.is_contiguous() and takes.is_contiguous() and grad_out.is_contiguous()):
        raise RuntimeError("backward inputs must be contiguous")
    num_nodes = _as_int64(num_nodes, "num_nodes")
    if num_nodes < 0:
        raise RuntimeError("num_nodes must be non-negative")
    B, D = grad_out.shape
    with _DeviceGuard(grad_out.device):
        stream = _stream_handle(grad_out.device)
        grad_x = _zeroed(num_nodes, D, grad_out.device, stream)
        if B == 0 or samples.size(1) == 0:
            return grad_x
        status = _L.fsa_sample_agg_backward(
            samples.data_ptr(), takes.data_ptr(), grad_out.data_ptr(), B, D, samples.size(1),
            grad_x.data_ptr(), num_nodes, stream)
        _lib.check(status, "fsa_sample_agg_backward")
    return grad_x


def _backward_2hop(grad_out, samples1, samples2, num_nodes, zeroed=None):
    if not (grad_out.is_cuda and samples1.is_cuda and samples2.is_cuda):
        raise RuntimeError("backward inputs must be CUDA tensors")
    if (grad_out.dtype != torch.float32 or samples1.dtype != torch.int32
            or samples2.dtype != torch.int32):
        raise RuntimeError("invalid backward input dtypes")
    if (grad_out.dim() != 2 or samples1.dim() != 2 or samples2.dim() != 3
            or samples1.size(0) != grad_out.size(0) or samples2.size(0) != grad_out.size(0)
            or samples2.size(1) != samples1.size(1)):
        raise RuntimeError("saved sample shapes do not match grad_out")
    if not (grad_out.device == samples1.device == samples2.device):
        raise RuntimeError("backward inputs must be on the same CUDA device")
    if not (grad_out.is_contiguous() and samples1.is_contiguous() and samples2.is_contiguous()):
        raise RuntimeError("backward inputs must be contiguous")
    num_nodes = _as_int64(num_nodes, "num_nodes")
    if num_nodes < 0:
        raise RuntimeError("num_nodes must be non-negative")
    B, D = grad_out.shape
    f1, f2 = samples1.size(1), samples2.size(2)
    with _DeviceGuard(grad_out.device):
        stream = _stream_handle(grad_out.device)
        grad_x = _grad_buffer(zeroed, num_nodes, D, grad_out.device, stream)
        if B == 0 or f1 == 0 or f2 == 0:
            return grad_x
        status = _L.fsa_sample_agg_2hop_backward(
            grad_out.data_ptr(), samples1.data_ptr(), samples2.data_ptr(), B, D, f1, f2,
            grad_x.data_ptr(), num_nodes, stream)
        _lib.check(status, "fsa_sample_agg_2hop_backward")
    return grad_x


# ---------------------------------------------------------------------------
# Public API (fuseop/__init__.py:75-206)
# ---------------------------------------------------------------------------

def fused_sample_agg(rowptr, col, x, frontier, fanout, replay_seed=1234, save_indices=False,
                     *, batch_offset=0):
    """Return the sampled 1-hop neighbor mean for each frontier node."""
    _check_python_inputs(rowptr, col, x, frontier)
    return _C.sample_agg(rowptr, col, x, frontier, _as_int64(fanout, "fanout"),
                         _as_seed(replay_seed), bool(save_indices),
                         _as_int64(batch_offset, "batch_offset"))


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
                          save_indices=False, *, batch_offset=0):
    """Return the nested sampled 2-hop neighbor mean for each frontier node."""
    _check_python_inputs(rowptr, col, x, frontier)
    return _C.sample_agg_2hop(rowptr, col, x, frontier, _as_int64(fanout1, "fanout1"),
                              _as_int64(fanout2, "fanout2"), _as_seed(replay_seed),
                              bool(save_indices), _as_int64(batch_offset, "batch_offset"))


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
