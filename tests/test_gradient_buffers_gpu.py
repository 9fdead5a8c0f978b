"""Gradient-buffer handling of the autograd path (GPU).

* The dense gradient that a 2-hop forward allocates ahead of its backward
  (so that the forward's draw kernel can zero it): at most one per feature
  table is pending, so k forwards before their backwards hold at most one
  extra N x D buffer -- the reference holds none until its backward
  allocates one (fuseop/binding.cpp:220).
* The opt-in PersistentGradient (``grad_buffer=``): the backward adds into
  a caller-held buffer that ``zero_()`` clears row by row; every step's
  gradient must equal the default path's fresh-zero gradient within
  rtol 1e-5 / atol 1e-6.
"""

from __future__ import annotations

import pytest
import torch

import fusesampleagg_b200 as fsa
from fusesampleagg_b200 import synthetic

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6


@pytest.fixture(scope="module")
def graph(cuda_device):
    g = synthetic.chung_lu_graph(200_000, 4_000_000, 2.1, 5_000, seed=5, device=cuda_device)
    return g.rowptr, g.col, g.num_nodes


def roots(n, b, seed):
    return synthetic.root_batch(n, b, seed, device="cuda")


def fresh_grad_2hop(rp, cl, x0, fr, go, seed, fan=(15, 10)):
    x = x0.detach().clone().requires_grad_(True)
    fsa.fused_sample_agg_2hop(rp, cl, x, fr, *fan, replay_seed=seed).backward(go)
    return x.grad


def fresh_grad_1hop(rp, cl, x0, fr, go, seed, k=10):
    x = x0.detach().clone().requires_grad_(True)
    fsa.fused_sample_agg(rp, cl, x, fr, k, replay_seed=seed).backward(go)
    return x.grad


# ---------------------------------------------------------------------------
# At most one forward-allocated gradient per table
# ---------------------------------------------------------------------------

def test_two_forwards_then_one_backward_hold_one_extra_buffer(graph):
    rp, cl, n = graph
    D = 64
    nd = n * D * 4
    x = synthetic.features(n, D, seed=1, device="cuda").requires_grad_(True)
    fr1, fr2 = roots(n, 512, 1), roots(n, 512, 2)
    go1 = synthetic.features(512, D, seed=3, device="cuda")
    go2 = synthetic.features(512, D, seed=4, device="cuda")
    want = fresh_grad_2hop(rp, cl, x, fr1, go1, 7) + fresh_grad_2hop(rp, cl, x, fr2, go2, 8)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    o1 = fsa.fused_sample_agg_2hop(rp, cl, x, fr1, 15, 10, replay_seed=7)
    o2 = fsa.fused_sample_agg_2hop(rp, cl, x, fr2, 15, 10, replay_seed=8)
    torch.cuda.synchronize()
    small = 8 << 20  # outputs, saved ids and workspaces of both calls
    held = torch.cuda.memory_allocated() - base
    assert nd <= held < nd + small, (held, nd)
    (o1 * go1).sum().add_((o2 * go2).sum()).backward()
    torch.cuda.synchronize()
    # the reference pattern: each backward's gradient, one accumulated into
    # the other (x.grad) -- two N x D at the peak (read before the comparison
    # below allocates its own temporaries)
    peak = torch.cuda.max_memory_allocated() - base
    assert peak < 2 * nd + small, (peak, nd)
    torch.testing.assert_close(x.grad, want, rtol=RTOL, atol=ATOL)


def test_single_forward_still_zeroes_its_gradient_in_the_forward(graph):
    rp, cl, n = graph
    D = 32
    x = synthetic.features(n, D, seed=1, device="cuda").requires_grad_(True)
    fr = roots(n, 256, 5)
    go = synthetic.features(256, D, seed=6, device="cuda")
    torch.cuda.synchronize()
    launches = fsa.launch_count()
    out = fsa.fused_sample_agg_2hop(rp, cl, x, fr, 15, 10, replay_seed=3)
    out.backward(go)
    torch.cuda.synchronize()
    # plan, draw (with the fill), gather, backward: no stand-alone fill kernel
    assert fsa.launch_count() - launches == 4
    torch.testing.assert_close(x.grad, fresh_grad_2hop(rp, cl, x, fr, go, 3), rtol=RTOL,
                               atol=ATOL)


def test_dropped_graph_releases_the_pending_buffer(graph):
    rp, cl, n = graph
    D = 16
    x = synthetic.features(n, D, seed=1, device="cuda").requires_grad_(True)
    fr = roots(n, 128, 9)
    out = fsa.fused_sample_agg_2hop(rp, cl, x, fr, 5, 5, replay_seed=1)
    del out  # graph and its buffer freed without a backward
    torch.cuda.synchronize()
    launches = fsa.launch_count()
    fsa.fused_sample_agg_2hop(rp, cl, x, fr, 5, 5, replay_seed=1).backward(
        torch.ones(128, D, device="cuda"))
    torch.cuda.synchronize()
    assert fsa.launch_count() - launches == 4  # the fill rode in the forward again


# ---------------------------------------------------------------------------
# PersistentGradient
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("hops", [1, 2])
def test_persistent_gradient_equals_fresh_gradient_every_step(graph, hops):
    rp, cl, n = graph
    D = 100
    x = synthetic.features(n, D, seed=1, device="cuda").requires_grad_(True)
    buf = fsa.PersistentGradient(x)
    assert torch.count_nonzero(buf.grad) == 0
    for step in range(4):
        fr = roots(n, 1024, 100 + step)
        go = synthetic.features(1024, D, seed=200 + step, device="cuda")
        buf.zero_()
        if hops == 2:
            out = fsa.fused_sample_agg_2hop(rp, cl, x, fr, 15, 10, replay_seed=step,
                                            grad_buffer=buf)
            want = fresh_grad_2hop(rp, cl, x, fr, go, step)
        else:
            out = fsa.fused_sample_agg(rp, cl, x, fr, 10, replay_seed=step, grad_buffer=buf)
            want = fresh_grad_1hop(rp, cl, x, fr, go, step)
        out.backward(go)
        assert x.grad is None  # the gradient went into the buffer, not through autograd
        torch.testing.assert_close(buf.grad, want, rtol=RTOL, atol=ATOL)


def test_persistent_gradient_output_is_the_default_paths(graph):
    rp, cl, n = graph
    x = synthetic.features(n, 24, seed=1, device="cuda").requires_grad_(True)
    buf = fsa.PersistentGradient(x)
    fr = roots(n, 300, 3)
    a = fsa.fused_sample_agg_2hop(rp, cl, x, fr, 8, 4, replay_seed=2, grad_buffer=buf)
    b = fsa.fused_sample_agg_2hop(rp, cl, x, fr, 8, 4, replay_seed=2)
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_persistent_gradient_accumulates_until_zeroed(graph):
    rp, cl, n = graph
    D = 40
    x = synthetic.features(n, D, seed=1, device="cuda").requires_grad_(True)
    buf = fsa.PersistentGradient(x)
    fr1, fr2 = roots(n, 512, 11), roots(n, 512, 12)
    go = synthetic.features(512, D, seed=13, device="cuda")
    fsa.fused_sample_agg_2hop(rp, cl, x, fr1, 15, 10, replay_seed=1, grad_buffer=buf).backward(go)
    fsa.fused_sample_agg_2hop(rp, cl, x, fr2, 15, 10, replay_seed=2, grad_buffer=buf).backward(go)
    want = fresh_grad_2hop(rp, cl, x, fr1, go, 1) + fresh_grad_2hop(rp, cl, x, fr2, go, 2)
    torch.testing.assert_close(buf.grad, want, rtol=RTOL, atol=ATOL)
    buf.zero_()
    assert torch.count_nonzero(buf.grad) == 0
    assert buf.pending_rows == 0


def test_zero_between_forward_and_backward(graph):
    rp, cl, n = graph
    D = 20
    x = synthetic.features(n, D, seed=1, device="cuda").requires_grad_(True)
    buf = fsa.PersistentGradient(x)
    go = synthetic.features(256, D, seed=14, device="cuda")
    fsa.fused_sample_agg_2hop(rp, cl, x, roots(n, 256, 20), 15, 10, replay_seed=5,
                              grad_buffer=buf).backward(go)
    fr = roots(n, 256, 21)
    out = fsa.fused_sample_agg_2hop(rp, cl, x, fr, 15, 10, replay_seed=6, grad_buffer=buf)
    buf.zero_()  # clears step 1's rows; this forward's stay recorded
    out.backward(go)
    torch.testing.assert_close(buf.grad, fresh_grad_2hop(rp, cl, x, fr, go, 6), rtol=RTOL,
                               atol=ATOL)
    buf.zero_()
    assert torch.count_nonzero(buf.grad) == 0


def test_dropped_graph_is_forgotten_by_zero(graph):
    rp, cl, n = graph
    x = synthetic.features(n, 8, seed=1, device="cuda").requires_grad_(True)
    buf = fsa.PersistentGradient(x)
    out = fsa.fused_sample_agg_2hop(rp, cl, x, roots(n, 64, 30), 4, 4, grad_buffer=buf)
    assert buf.pending_rows == 64 * 16
    buf.zero_()
    assert buf.pending_rows == 64 * 16  # its backward may still run
    del out
    buf.zero_()
    assert buf.pending_rows == 0


def test_persistent_gradient_without_grad_records_nothing(graph):
    rp, cl, n = graph
    x = synthetic.features(n, 8, seed=1, device="cuda").requires_grad_(True)
    buf = fsa.PersistentGradient(x)
    with torch.no_grad():
        out = fsa.fused_sample_agg_2hop(rp, cl, x, roots(n, 64, 31), 4, 4, grad_buffer=buf)
    assert out.grad_fn is None and buf.pending_rows == 0


def test_persistent_gradient_argument_checks(graph):
    rp, cl, n = graph
    x = synthetic.features(n, 8, seed=1, device="cuda").requires_grad_(True)
    fr = roots(n, 8, 1)
    with pytest.raises(TypeError, match="PersistentGradient"):
        fsa.fused_sample_agg_2hop(rp, cl, x, fr, 2, 2, grad_buffer=torch.zeros_like(x))
    other = fsa.PersistentGradient(synthetic.features(n, 9, seed=1, device="cuda"))
    with pytest.raises(RuntimeError, match="grad_buffer shape must equal the features' shape"):
        fsa.fused_sample_agg_2hop(rp, cl, x, fr, 2, 2, grad_buffer=other)
    with pytest.raises(ValueError, match="2-D CUDA feature tensor"):
        fsa.PersistentGradient(x.detach().cpu())


@pytest.mark.parametrize("hops", [1, 2])
def test_clear_inside_the_call_equals_zero_then_call(graph, hops):
    """clear_grad_buffer=True: the recorded rows are zeroed as part of the
    call (for 2-hop inside the sampling kernel); every step's buffer equals
    the default path's fresh gradient."""
    rp, cl, n = graph
    D = 100
    x = synthetic.features(n, D, seed=1, device="cuda").requires_grad_(True)
    buf = fsa.PersistentGradient(x)
    for step in range(4):
        fr = roots(n, 1024, 300 + step)
        go = synthetic.features(1024, D, seed=400 + step, device="cuda")
        torch.cuda.synchronize()
        launches = fsa.launch_count()
        if hops == 2:
            out = fsa.fused_sample_agg_2hop(rp, cl, x, fr, 15, 10, replay_seed=step,
                                            grad_buffer=buf, clear_grad_buffer=True)
        else:
            out = fsa.fused_sample_agg(rp, cl, x, fr, 10, replay_seed=step, grad_buffer=buf,
                                       clear_grad_buffer=True)
        out.backward(go)
        torch.cuda.synchronize()
        if hops == 2:
            # plan, draw (with the row clear), gather, backward
            assert fsa.launch_count() - launches == 4
        want = (fresh_grad_2hop(rp, cl, x, fr, go, step) if hops == 2
                else fresh_grad_1hop(rp, cl, x, fr, go, step))
        torch.testing.assert_close(buf.grad, want, rtol=RTOL, atol=ATOL)
    with pytest.raises(ValueError, match="needs a grad_buffer"):
        fsa.fused_sample_agg_2hop(rp, cl, x, roots(n, 8, 1), 2, 2, clear_grad_buffer=True)


@pytest.mark.parametrize("dim", [100, 37, 256])
def test_forward_zero_rows_entry_point(graph, dim):
    """fsa_sample_agg_2hop_forward_zero_rows through the C ABI: the listed rows
    (with -1 padding and out-of-range entries) of the table are zero, all
    other rows unchanged, and the forward's outputs are those of the plain
    entry point.  D = 100 clears inside the draw kernel; D = 37 and 256 take
    the stand-alone row kernel first."""
    from fusesampleagg_b200 import _lib

    L = _lib.LIB
    rp, cl, n = graph
    x = synthetic.features(n, dim, seed=1, device="cuda")
    fr = roots(n, 512, 7)
    B, k1, k2 = 512, 15, 10
    table = torch.ones((n, dim), device="cuda")
    rows = torch.randint(0, n, (3000,), dtype=torch.int32, device="cuda")
    rows[::7] = -1
    rows[::11] = n + 5
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for clear in (False, True):
        out = torch.empty((B, dim), device="cuda")
        s1 = torch.empty((B, k1), dtype=torch.int32, device="cuda")
        s2 = torch.empty((B, k1, k2), dtype=torch.int32, device="cuda")
        nbytes = L.fsa_sample_agg_2hop_workspace_size(B, k1, k2, 1, 1)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        head = (rp.data_ptr(), cl.data_ptr(), n, cl.numel(), x.data_ptr(), dim, fr.data_ptr(), B,
                0, k1, k2, 9, out.data_ptr(), s1.data_ptr(), s2.data_ptr(), ws.data_ptr(), nbytes)
        if clear:
            st = L.fsa_sample_agg_2hop_forward_zero_rows(*head, table.data_ptr(), rows.data_ptr(),
                                                         rows.numel(), stream)
        else:
            st = L.fsa_sample_agg_2hop_forward(*head, None, 0, stream)
        _lib.check(st, "2-hop forward")
        outs.append((out, s1, s2))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0].view(torch.int32), outs[1][0].view(torch.int32))
    assert torch.equal(outs[0][2], outs[1][2])
    valid = rows[(rows >= 0) & (rows < n)].long()
    mask = torch.zeros(n, dtype=torch.bool, device="cuda")
    mask[valid] = True
    assert torch.count_nonzero(table[mask]) == 0
    assert bool((table[~mask] == 1).all())
