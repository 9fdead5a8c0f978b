"""The error contract on the path that raises it (GPU).

Every check of the reference binding -- graph inputs and fanouts
(fuseop/binding.cpp:16-53), the 1-hop backward (:119-135) and the 2-hop
backward (:200-218) -- is asserted here with its exception type and message,
through the public functions where they reach it and otherwise through the
binding's entry points (``fusesampleagg_b200._C``), which are the
counterparts of the reference's ``fuseop._C`` functions.  The Python-side
ValueError / TypeError checks (fuseop/__init__.py:15-29) are asserted with
real CUDA tensors too.

Two conditions are not reachable on one GPU or through any public call:
"all inputs must be on the same CUDA device" needs a second device (tested
when one is present), and "all inputs must be contiguous" never fires for
the forward because, as in the reference's public API
(fuseop/__init__.py:50-58), inputs are made contiguous before the check.
"""

from __future__ import annotations

import pytest
import torch

import fusesampleagg_b200 as fsa

pytestmark = pytest.mark.gpu

C = fsa._C


@pytest.fixture(scope="module")
def g(cuda_device):
    dev = cuda_device
    return {
        "rowptr": torch.tensor([0, 2, 3, 4], dtype=torch.int32, device=dev),
        "col": torch.tensor([1, 2, 0, 1], dtype=torch.int32, device=dev),
        "x": torch.randn(3, 8, device=dev),
        "frontier": torch.tensor([0, 2], dtype=torch.int32, device=dev),
    }


def call(fn, g, *fan, **over):
    a = dict(g)
    a.update(over)
    return fn(a["rowptr"], a["col"], a["x"], a["frontier"], *fan)


PUBLIC = [
    (fsa.fused_sample_agg, (2,)),
    (fsa.fused_sample_agg_with_samples, (2,)),
    (fsa.fused_sample_agg_2hop, (2, 2)),
    (fsa.fused_sample_agg_2hop_with_samples, (2, 2)),
]


# ---------------------------------------------------------------------------
# Python-side checks (fuseop/__init__.py:15-29)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("fn,fan", PUBLIC)
def test_cpu_input_is_value_error(g, fn, fan):
    with pytest.raises(ValueError, match="rowptr, col, x, and frontier must be CUDA tensors"):
        call(fn, g, *fan, frontier=g["frontier"].cpu())


@pytest.mark.parametrize("fn,fan", PUBLIC)
@pytest.mark.parametrize("field,dtype,msg", [
    ("rowptr", torch.int64, "rowptr and col must have dtype torch.int32"),
    ("col", torch.int64, "rowptr and col must have dtype torch.int32"),
    ("frontier", torch.int64, "frontier must have dtype torch.int32"),
    ("x", torch.float64, "x must have dtype torch.float32"),
])
def test_wrong_dtype_is_type_error(g, fn, fan, field, dtype, msg):
    with pytest.raises(TypeError, match=msg):
        call(fn, g, *fan, **{field: g[field].to(dtype)})


# ---------------------------------------------------------------------------
# Graph-input checks (fuseop/binding.cpp:16-37)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("fn,fan", PUBLIC)
@pytest.mark.parametrize("over", [
    lambda g: {"x": g["x"].reshape(-1)},
    lambda g: {"rowptr": g["rowptr"].reshape(2, 2)},
    lambda g: {"col": g["col"].reshape(2, 2)},
    lambda g: {"frontier": g["frontier"].reshape(1, 2)},
])
def test_wrong_rank_is_runtime_error(g, fn, fan, over):
    with pytest.raises(RuntimeError, match=r"expected rowptr\[N\+1\], col\[E\], x\[N,D\], "
                                           r"and frontier\[B\]"):
        call(fn, g, *fan, **over(g))


@pytest.mark.parametrize("fn,fan", PUBLIC)
def test_rowptr_length_is_runtime_error(g, fn, fan):
    with pytest.raises(RuntimeError, match=r"rowptr length must equal N\+1"):
        call(fn, g, *fan, rowptr=g["rowptr"][:3].contiguous())


def binding_forwards():
    # the binding's forward entry points: (fn, trailing args after the four
    # tensors) -- seed, capture flag / batch offset as each takes them
    return [
        (C.sample_agg, (2, 1, False, 0)),
        (C.sample_agg_with_samples, (2, 1, 0)),
        (C.sample_agg_2hop, (2, 2, 1, False, 0)),
        (C.sample_agg_2hop_with_samples, (2, 2, 1, 0)),
    ]


@pytest.mark.parametrize("k", range(4))
def test_binding_rejects_cpu_inputs(g, k):
    fn, rest = binding_forwards()[k]
    with pytest.raises(RuntimeError, match="all inputs must be CUDA tensors"):
        call(fn, g, *rest, col=g["col"].cpu())


@pytest.mark.parametrize("k", range(4))
@pytest.mark.parametrize("field,dtype,msg", [
    ("rowptr", torch.int64, "rowptr, col, and frontier must be int32"),
    ("col", torch.int16, "rowptr, col, and frontier must be int32"),
    ("frontier", torch.int64, "rowptr, col, and frontier must be int32"),
    ("x", torch.float16, "x must be float32"),
])
def test_binding_rejects_wrong_dtypes(g, k, field, dtype, msg):
    fn, rest = binding_forwards()[k]
    with pytest.raises(RuntimeError, match=msg):
        call(fn, g, *rest, **{field: g[field].to(dtype)})


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second CUDA device")
@pytest.mark.parametrize("fn,fan", PUBLIC)
def test_inputs_on_two_devices_is_runtime_error(g, fn, fan):
    with pytest.raises(RuntimeError, match="all inputs must be on the same CUDA device"):
        call(fn, g, *fan, frontier=g["frontier"].to("cuda:1"))


def test_non_contiguous_inputs_are_accepted(g):
    # the reference's public functions pass .contiguous() copies to the
    # binding (fuseop/__init__.py:50-58); so does this package
    fr = torch.tensor([0, 9, 2, 9], dtype=torch.int32, device=g["x"].device)[::2]
    assert not fr.is_contiguous()
    a = fsa.fused_sample_agg_2hop(g["rowptr"], g["col"], g["x"], fr, 2, 2)
    b = fsa.fused_sample_agg_2hop(g["rowptr"], g["col"], g["x"], fr.contiguous(), 2, 2)
    assert torch.equal(a, b)


# ---------------------------------------------------------------------------
# Fanout checks (fuseop/binding.cpp:39-53)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("fn", [fsa.fused_sample_agg, fsa.fused_sample_agg_with_samples])
@pytest.mark.parametrize("fanout,msg", [(-1, "fanout must be non-negative"),
                                        (1025, "fanout exceeds the supported maximum of 1024")])
def test_1hop_fanout_limits(g, fn, fanout, msg):
    with pytest.raises(RuntimeError, match=msg):
        call(fn, g, fanout)
    call(fn, g, 1024)  # the limit itself is accepted


@pytest.mark.parametrize("fn", [fsa.fused_sample_agg_2hop, fsa.fused_sample_agg_2hop_with_samples])
@pytest.mark.parametrize("f1,f2,msg", [
    (-1, 2, "fanouts must be non-negative"),
    (2, -1, "fanouts must be non-negative"),
    (2, 2**62, "fanout pair is too large"),
    (1000, 12, "fanout pair requires too much shared memory; reduce fanout1 or fanout2"),
])
def test_2hop_fanout_limits(g, fn, f1, f2, msg):
    with pytest.raises(RuntimeError, match=msg):
        call(fn, g, f1, f2)
    call(fn, g, 1000, 11)  # 1000 + 1000 * 11 = 12000 entries: accepted


# ---------------------------------------------------------------------------
# Backward checks (fuseop/binding.cpp:119-135 and :200-218), through the
# binding's replay entry points
# ---------------------------------------------------------------------------

@pytest.fixture(scope="module")
def saved(g):
    _, samples, takes = fsa.fused_sample_agg_with_samples(g["rowptr"], g["col"], g["x"],
                                                           g["frontier"], 2)
    _, s1, s2 = fsa.fused_sample_agg_2hop_with_samples(g["rowptr"], g["col"], g["x"],
                                                        g["frontier"], 2, 2)
    go = torch.randn(2, 8, device=g["x"].device)
    return {"samples": samples, "takes": takes, "s1": s1, "s2": s2, "go": go}


def bwd1(sv, **over):
    a = {"samples": sv["samples"], "takes": sv["takes"], "go": sv["go"], "n": 3}
    a.update(over)
    return C.sample_agg_backward(a["samples"], a["takes"], a["go"], a["n"])


def bwd2(sv, **over):
    a = {"go": sv["go"], "s1": sv["s1"], "s2": sv["s2"], "n": 3}
    a.update(over)
    return C.sample_agg_2hop_backward(a["go"], a["s1"], a["s2"], a["n"])


@pytest.mark.parametrize("over,msg", [
    (lambda s: {"takes": s["takes"].cpu()}, "backward inputs must be CUDA tensors"),
    (lambda s: {"samples": s["samples"].long()}, "samples and takes must be int32"),
    (lambda s: {"takes": s["takes"].long()}, "samples and takes must be int32"),
    (lambda s: {"go": s["go"].double()}, "grad_out must be a float32 matrix"),
    (lambda s: {"go": s["go"].reshape(-1)}, "grad_out must be a float32 matrix"),
    (lambda s: {"samples": s["samples"][:1]}, "saved sample shapes do not match grad_out"),
    (lambda s: {"takes": s["takes"][:1]}, "saved sample shapes do not match grad_out"),
    (lambda s: {"samples": s["samples"].reshape(-1)}, "saved sample shapes do not match grad_out"),
    (lambda s: {"go": s["go"].t().contiguous().t()}, "backward inputs must be contiguous"),
    (lambda s: {"n": -1}, "num_nodes must be non-negative"),
])
def test_1hop_backward_checks(saved, over, msg):
    with pytest.raises(RuntimeError, match=msg):
        bwd1(saved, **over(saved))


@pytest.mark.parametrize("over,msg", [
    (lambda s: {"s2": s["s2"].cpu()}, "backward inputs must be CUDA tensors"),
    (lambda s: {"go": s["go"].double()}, "invalid backward input dtypes"),
    (lambda s: {"s1": s["s1"].long()}, "invalid backward input dtypes"),
    (lambda s: {"s2": s["s2"].long()}, "invalid backward input dtypes"),
    (lambda s: {"go": s["go"].reshape(-1)}, "saved sample shapes do not match grad_out"),
    (lambda s: {"s1": s["s1"][:1]}, "saved sample shapes do not match grad_out"),
    (lambda s: {"s2": s["s2"][:1]}, "saved sample shapes do not match grad_out"),
    (lambda s: {"s2": s["s2"][:, :1].contiguous()}, "saved sample shapes do not match grad_out"),
    (lambda s: {"s2": s["s2"].reshape(2, -1)}, "saved sample shapes do not match grad_out"),
    (lambda s: {"go": s["go"].t().contiguous().t()}, "backward inputs must be contiguous"),
    (lambda s: {"n": -1}, "num_nodes must be non-negative"),
])
def test_2hop_backward_checks(saved, over, msg):
    with pytest.raises(RuntimeError, match=msg):
        bwd2(saved, **over(saved))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second CUDA device")
def test_backward_inputs_on_two_devices(saved):
    with pytest.raises(RuntimeError, match="backward inputs must be on the same CUDA device"):
        bwd1(saved, takes=saved["takes"].to("cuda:1"))
    with pytest.raises(RuntimeError, match="backward inputs must be on the same CUDA device"):
        bwd2(saved, s2=saved["s2"].to("cuda:1"))


def test_backward_replays_match_autograd(g, saved):
    """The replay entry points give the autograd backward's gradient."""
    x = g["x"].clone().requires_grad_(True)
    fsa.fused_sample_agg(g["rowptr"], g["col"], x, g["frontier"], 2).backward(saved["go"])
    torch.testing.assert_close(bwd1(saved), x.grad, rtol=1e-5, atol=1e-6)
    x.grad = None
    fsa.fused_sample_agg_2hop(g["rowptr"], g["col"], x, g["frontier"], 2, 2).backward(saved["go"])
    torch.testing.assert_close(bwd2(saved), x.grad, rtol=1e-5, atol=1e-6)
