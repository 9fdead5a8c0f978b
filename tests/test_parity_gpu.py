"""Parity of the sm_100a operator with the CPU oracle (bit-exact ids and
forward outputs, fp32-tolerance gradients) on the golden-case graphs.

Tolerance for gradients: rtol 1e-5, atol 1e-6 (fp32 atomics accumulate in a
different order than the oracle's sequential loop).
"""

from __future__ import annotations

import functools

import numpy as np
import pytest
import torch

import fusesampleagg_b200 as fsa
from fusesampleagg_b200 import synthetic
from oracle import oracle
from tests.golden import cases as C

pytestmark = pytest.mark.gpu

U64_MAX = (1 << 64) - 1
RTOL, ATOL = 1e-5, 1e-6


@functools.lru_cache(maxsize=None)
def cpu_graph(name):
    return C.GRAPHS[name]()


@functools.lru_cache(maxsize=None)
def dev_graph(name):
    g = cpu_graph(name)
    return g.rowptr.cuda(), g.col.cuda()


@functools.lru_cache(maxsize=None)
def cpu_features(n, d, seed=1):
    return synthetic.features(n, d, seed=seed)


def frontier(name, batch=64, seed=0):
    return C.frontier_for(name, cpu_graph(name), batch, seed)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().numpy().view(np.int32)


def assert_bit_equal(mine: torch.Tensor, ref: np.ndarray):
    ref = np.ascontiguousarray(ref, dtype=np.float32)
    got = mine.detach().cpu().numpy()
    if not np.array_equal(got.view(np.int32), ref.view(np.int32)):
        diff = np.abs(got - ref)
        raise AssertionError(f"not bit-identical: max |diff| {diff.max()} at {np.unravel_index(diff.argmax(), diff.shape)}")


def run_1hop(name, k, seed, dim=33, batch=64, root_seed=0, offset=0):
    g = cpu_graph(name)
    rp, cl = dev_graph(name)
    x = cpu_features(g.num_nodes, dim)
    fr = frontier(name, batch, root_seed)
    out, samples, takes = fsa.fused_sample_agg_with_samples(
        rp, cl, x.cuda(), fr.cuda(), k, replay_seed=seed, batch_offset=offset)
    ref_s, ref_t = oracle.sample_1hop(g.rowptr.numpy(), g.col.numpy(), fr.numpy(), k, seed,
                                      batch_offset=offset)
    ref_out = oracle.forward_1hop(x.numpy(), ref_s, ref_t)
    return out, samples, takes, ref_out, ref_s, ref_t


def run_2hop(name, k1, k2, seed, dim=33, batch=64, root_seed=0, offset=0):
    g = cpu_graph(name)
    rp, cl = dev_graph(name)
    x = cpu_features(g.num_nodes, dim)
    fr = frontier(name, batch, root_seed)
    out, s1, s2 = fsa.fused_sample_agg_2hop_with_samples(
        rp, cl, x.cuda(), fr.cuda(), k1, k2, replay_seed=seed, batch_offset=offset)
    r1, r2 = oracle.sample_2hop(g.rowptr.numpy(), g.col.numpy(), fr.numpy(), k1, k2, seed,
                                batch_offset=offset)
    ref_out = oracle.forward_2hop(x.numpy(), r2)
    return out, s1, s2, ref_out, r1, r2


def test_large_batch_uses_scan_kernel_and_matches_oracle():
    """2048+ roots: the root prefix no longer fits the draw kernel's shared
    memory and a separate scan kernel runs (plan, scan, draws, gather)."""
    g = cpu_graph("uniform")
    rp, cl = dev_graph("uniform")
    x = cpu_features(g.num_nodes, 8)
    fr = C.frontier_for("uniform", g, 3000, 9)
    before = fsa.launch_count()
    out, s1, s2 = fsa.fused_sample_agg_2hop_with_samples(rp, cl, x.cuda(), fr.cuda(), 5, 4,
                                                         replay_seed=21)
    assert fsa.launch_count() == before + 4
    r1, r2 = oracle.sample_2hop(g.rowptr.numpy(), g.col.numpy(), fr.numpy(), 5, 4, 21)
    np.testing.assert_array_equal(s1.cpu().numpy(), r1)
    np.testing.assert_array_equal(s2.cpu().numpy(), r2)
    assert_bit_equal(out, oracle.forward_2hop(x.numpy(), r2))


# ---------------------------------------------------------------------------
# 1-hop
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", ["toy", "hub", "uniform", "powerlaw"])
@pytest.mark.parametrize("k", [0, 1, 2, 5, 10, 11, 64, 1024])
@pytest.mark.parametrize("seed", [0, 17, U64_MAX])
def test_1hop_ids_and_outputs_bit_exact(name, k, seed):
    out, samples, takes, ref_out, ref_s, ref_t = run_1hop(name, k, seed)
    np.testing.assert_array_equal(samples.cpu().numpy(), ref_s)
    np.testing.assert_array_equal(takes.cpu().numpy(), ref_t)
    assert_bit_equal(out, ref_out)


@pytest.mark.parametrize("dim", [1, 2, 3, 4, 8, 31, 32, 33, 64, 100, 127, 128, 129, 256, 602])
def test_1hop_feature_widths(dim):
    out, _, _, ref_out, _, _ = run_1hop("powerlaw", 10, 5, dim=dim, batch=128)
    assert_bit_equal(out, ref_out)


def test_1hop_no_capture_matches_capture():
    g = cpu_graph("powerlaw")
    rp, cl = dev_graph("powerlaw")
    x = cpu_features(g.num_nodes, 100).cuda()
    fr = frontier("powerlaw", 256, 3).cuda()
    a = fsa.fused_sample_agg(rp, cl, x, fr, 10, replay_seed=3)
    b, _, _ = fsa.fused_sample_agg_with_samples(rp, cl, x, fr, 10, replay_seed=3)
    assert torch.equal(bits_t(a), bits_t(b))


def bits_t(t):
    return t.contiguous().view(torch.int32)


@pytest.mark.parametrize("name,k", [("toy", 3), ("powerlaw", 10), ("hub", 11), ("uniform", 1024)])
def test_1hop_backward_matches_oracle(name, k):
    g = cpu_graph(name)
    rp, cl = dev_graph(name)
    x = cpu_features(g.num_nodes, 19).cuda().requires_grad_(True)
    fr = frontier(name, 96, 1)
    out = fsa.fused_sample_agg(rp, cl, x, fr.cuda(), k, replay_seed=42)
    go = synthetic.features(out.size(0), 19, seed=2)
    out.backward(go.cuda())
    s, t = oracle.sample_1hop(g.rowptr.numpy(), g.col.numpy(), fr.numpy(), k, 42)
    ref = oracle.backward_1hop(s, t, go.numpy(), g.num_nodes)
    np.testing.assert_allclose(x.grad.cpu().numpy(), ref, rtol=RTOL, atol=ATOL)


# ---------------------------------------------------------------------------
# 2-hop
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", ["toy", "hub", "uniform", "powerlaw"])
@pytest.mark.parametrize("fan", [(1, 1), (3, 2), (5, 10), (15, 10), (25, 10), (8, 4), (2, 100)])
@pytest.mark.parametrize("seed", [0, 1234, U64_MAX])
def test_2hop_ids_and_outputs_bit_exact(name, fan, seed):
    out, s1, s2, ref_out, r1, r2 = run_2hop(name, *fan, seed)
    np.testing.assert_array_equal(s1.cpu().numpy(), r1)
    np.testing.assert_array_equal(s2.cpu().numpy(), r2)
    assert_bit_equal(out, ref_out)


@pytest.mark.parametrize("name", ["powerlaw", "hub", "uniform"])
@pytest.mark.parametrize("seed", [3, U64_MAX])
def test_hub_roots_bit_exact(name, seed):
    """Roots = the highest-degree nodes: every first-hop row is long and the
    first-hop draws of a root are spread over the whole CTA."""
    out, s1, s2, ref_out, r1, r2 = run_2hop(name, 15, 10, seed, root_seed=-1, batch=96)
    np.testing.assert_array_equal(s1.cpu().numpy(), r1)
    np.testing.assert_array_equal(s2.cpu().numpy(), r2)
    assert_bit_equal(out, ref_out)
    out, s, t, ref_out, rs, rt = run_1hop(name, 10, seed, root_seed=-1, batch=96)
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    assert_bit_equal(out, ref_out)


@pytest.mark.parametrize("dim", [1, 2, 3, 4, 8, 16, 33, 64, 100, 127, 128, 129, 256, 602, 1000])
def test_2hop_feature_widths(dim):
    out, _, _, ref_out, _, _ = run_2hop("powerlaw", 15, 10, 7, dim=dim, batch=64)
    assert_bit_equal(out, ref_out)


@pytest.mark.parametrize("fan", [(0, 0), (0, 2), (2, 0)])
def test_2hop_zero_fanout_returns_zero(fan):
    rp, cl = dev_graph("toy")
    x = cpu_features(8, 16).cuda()
    fr = frontier("toy").cuda()
    out, s1, s2 = fsa.fused_sample_agg_2hop_with_samples(rp, cl, x, fr, *fan, replay_seed=1)
    assert torch.count_nonzero(out) == 0
    assert bool((s1 == -1).all()) and bool((s2 == -1).all())
    assert tuple(s1.shape) == (fr.numel(), fan[0]) and tuple(s2.shape) == (fr.numel(), *fan)


def test_empty_frontier():
    rp, cl = dev_graph("toy")
    x = cpu_features(8, 16).cuda()
    fr = torch.empty(0, dtype=torch.int32, device="cuda")
    assert fsa.fused_sample_agg(rp, cl, x, fr, 3).shape == (0, 16)
    assert fsa.fused_sample_agg_2hop(rp, cl, x, fr, 3, 2).shape == (0, 16)


def test_phase_timing_records_each_forward_kernel():
    from fusesampleagg_b200 import _lib

    _lib.phase_timing(True)
    try:
        out, s1, s2, ref_out, r1, r2 = run_2hop("powerlaw", 15, 10, 3, batch=64)
        run_2hop("powerlaw", 15, 10, 4, batch=64)
        times, calls = _lib.phase_times()
    finally:
        _lib.phase_timing(False)
    assert calls == 2
    assert all(v > 0.0 for v in times.values()), times
    np.testing.assert_array_equal(s2.cpu().numpy(), r2)
    # recording stopped: later forwards add nothing
    run_2hop("powerlaw", 15, 10, 5, batch=64)
    assert _lib.phase_times()[1] == 0


@pytest.mark.parametrize("name,fan", [("toy", (3, 2)), ("powerlaw", (15, 10)), ("hub", (5, 10)),
                                      ("powerlaw", (8, 4))])
def test_2hop_backward_matches_oracle(name, fan):
    g = cpu_graph(name)
    rp, cl = dev_graph(name)
    x = cpu_features(g.num_nodes, 20).cuda().requires_grad_(True)
    fr = frontier(name, 128, 2)
    out = fsa.fused_sample_agg_2hop(rp, cl, x, fr.cuda(), *fan, replay_seed=7)
    go = synthetic.features(out.size(0), 20, seed=2)
    out.backward(go.cuda())
    r1, r2 = oracle.sample_2hop(g.rowptr.numpy(), g.col.numpy(), fr.numpy(), *fan, 7)
    ref = oracle.backward_2hop(go.numpy(), r1, r2, g.num_nodes)
    np.testing.assert_allclose(x.grad.cpu().numpy(), ref, rtol=RTOL, atol=ATOL)


# ---------------------------------------------------------------------------
# API behaviour shared by both hops
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("hops", [1, 2])
def test_batch_offset_reproduces_slice_of_whole_batch(hops):
    g = cpu_graph("powerlaw")
    rp, cl = dev_graph("powerlaw")
    x = cpu_features(g.num_nodes, 8).cuda()
    fr = frontier("powerlaw", 200, 6).cuda()
    for off in (0, 1, 77, 199):
        if hops == 1:
            whole = fsa.fused_sample_agg_with_samples(rp, cl, x, fr, 10, replay_seed=5)
            part = fsa.fused_sample_agg_with_samples(rp, cl, x, fr[off:], 10, replay_seed=5,
                                                     batch_offset=off)
        else:
            whole = fsa.fused_sample_agg_2hop_with_samples(rp, cl, x, fr, 15, 10, replay_seed=5)
            part = fsa.fused_sample_agg_2hop_with_samples(rp, cl, x, fr[off:], 15, 10,
                                                          replay_seed=5, batch_offset=off)
        for w, p in zip(whole, part):
            assert torch.equal(w[off:].contiguous().view(torch.int32), p.contiguous().view(torch.int32))


def test_seed_and_frontier_order_are_reproducible():
    rp, cl = dev_graph("hub")
    g = cpu_graph("hub")
    x = cpu_features(g.num_nodes, 16).cuda()
    fr = frontier("hub", 64, 0).cuda()
    a = fsa.fused_sample_agg_2hop_with_samples(rp, cl, x, fr, 15, 10, 99)
    b = fsa.fused_sample_agg_2hop_with_samples(rp, cl, x, fr, 15, 10, 99)
    for lhs, rhs in zip(a, b):
        assert torch.equal(lhs, rhs)


@pytest.mark.parametrize("hops", [1, 2])
def test_non_default_stream(hops):
    g = cpu_graph("powerlaw")
    rp, cl = dev_graph("powerlaw")
    x = cpu_features(g.num_nodes, 129).cuda()
    fr = frontier("powerlaw", 64, 0).cuda()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        if hops == 1:
            out = fsa.fused_sample_agg(rp, cl, x, fr, 10, replay_seed=5)
        else:
            out = fsa.fused_sample_agg_2hop(rp, cl, x, fr, 15, 10, replay_seed=5)
        marker = out.square().sum()
    stream.synchronize()
    assert torch.isfinite(marker)
    ref = (fsa.fused_sample_agg(rp, cl, x, fr, 10, replay_seed=5) if hops == 1
           else fsa.fused_sample_agg_2hop(rp, cl, x, fr, 15, 10, replay_seed=5))
    assert torch.equal(out, ref)


def test_save_indices_without_grad_still_replays():
    g = cpu_graph("toy")
    rp, cl = dev_graph("toy")
    x = cpu_features(8, 12).cuda()
    out = fsa.fused_sample_agg_2hop(rp, cl, x, frontier("toy").cuda(), 3, 2, replay_seed=3,
                                    save_indices=True)
    assert out.shape == (9, 12) and not out.requires_grad


def test_launch_count_advances():
    rp, cl = dev_graph("toy")
    x = cpu_features(8, 12).cuda()
    before = fsa.launch_count()
    fsa.fused_sample_agg_2hop(rp, cl, x, frontier("toy").cuda(), 3, 2)
    # plan, draws (the root prefix is scanned in the draw kernel), gather
    assert fsa.launch_count() == before + 3
    before = fsa.launch_count()
    fsa.fused_sample_agg(rp, cl, x, frontier("toy").cuda(), 3)
    assert fsa.launch_count() == before + 1


# ---------------------------------------------------------------------------
# Out-of-range ids are skipped and reported, never dereferenced
# ---------------------------------------------------------------------------

def test_bad_root_is_flagged_and_row_left_empty():
    g = cpu_graph("powerlaw")
    rp, cl = dev_graph("powerlaw")
    x = cpu_features(g.num_nodes, 8)
    fr = frontier("powerlaw", 16, 0).clone()
    fr[3] = -1
    fr[7] = g.num_nodes
    fsa.device_status(reset=True)
    out, s, t = fsa.fused_sample_agg_with_samples(rp, cl, x.cuda(), fr.cuda(), 10, replay_seed=2)
    flags = fsa.device_status(reset=True)
    assert flags & 0x1
    assert int(t[3]) == 0 and int(t[7]) == 0
    assert torch.count_nonzero(out[3]) == 0 and torch.count_nonzero(out[7]) == 0
    for b in (0, 5, 15):
        rs, rt = oracle.sample_1hop(g.rowptr.numpy(), g.col.numpy(), fr[b:b + 1].numpy(), 10, 2,
                                    batch_offset=b)
        np.testing.assert_array_equal(s[b:b + 1].cpu().numpy(), rs)


def test_bad_neighbor_and_bad_row_are_flagged():
    # Row 0 -> [1, 9 (out of range)], row 1 -> [0], row 2: rowptr decreasing.
    rowptr = torch.tensor([0, 2, 3, 1, 3], dtype=torch.int32, device="cuda")
    col = torch.tensor([1, 9, 0], dtype=torch.int32, device="cuda")
    x = torch.arange(8, dtype=torch.float32, device="cuda").reshape(4, 2)
    fr = torch.tensor([0, 2, 1], dtype=torch.int32, device="cuda")
    fsa.device_status(reset=True)
    out, s1, s2 = fsa.fused_sample_agg_2hop_with_samples(rowptr, col, x, fr, 2, 2, replay_seed=1)
    flags = fsa.device_status(reset=True)
    assert flags & 0x2 and flags & 0x4
    assert torch.isfinite(out).all()


# ---------------------------------------------------------------------------
# Sort-by-destination backward (alternative to the atomic scatter)
# ---------------------------------------------------------------------------

def atomic_backward(go, s1, s2, num_nodes, base=None):
    """The step's backward (red.global.add) through the C ABI, adding into
    `base` (a copy) or into zeros."""
    from fusesampleagg_b200 import _lib

    B, D = go.shape
    grad = (base.clone() if base is not None
            else torch.zeros((num_nodes, D), device=go.device))
    _lib.check(_lib.LIB.fsa_sample_agg_2hop_backward(
        go.data_ptr(), s1.data_ptr(), s2.data_ptr(), B, D, s1.size(1), s2.size(2),
        grad.data_ptr(), num_nodes, torch.cuda.current_stream().cuda_stream), "backward")
    return grad


def sorted_backward(go, s1, s2, num_nodes, base=None):
    from fusesampleagg_b200 import _lib

    L = _lib.LIB
    B, D = go.shape
    k1, k2 = s1.size(1), s2.size(2)
    grad = (base.clone() if base is not None
            else torch.zeros((num_nodes, D), device=go.device))
    nbytes = L.fsa_sample_agg_2hop_backward_sorted_workspace_size(num_nodes, B, k1, k2)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=go.device)
    _lib.check(L.fsa_sample_agg_2hop_backward_sorted(
        go.data_ptr(), s1.data_ptr(), s2.data_ptr(), B, D, k1, k2, grad.data_ptr(), num_nodes,
        ws.data_ptr(), nbytes, torch.cuda.current_stream().cuda_stream), "sorted backward")
    return grad


@pytest.mark.parametrize("name,fan,dim", [("toy", (3, 2), 19), ("powerlaw", (15, 10), 100),
                                          ("hub", (5, 10), 33), ("powerlaw", (8, 4), 2),
                                          ("uniform", (25, 10), 64)])
def test_sorted_backward_matches_oracle(name, fan, dim):
    g = cpu_graph(name)
    out, s1, s2, _, r1, r2 = run_2hop(name, fan[0], fan[1], 7, dim=dim, batch=96)
    go = synthetic.features(s1.size(0), dim, seed=4)
    grad = sorted_backward(go.cuda(), s1, s2, g.num_nodes)
    ref = oracle.backward_2hop(go.numpy(), r1, r2, g.num_nodes)
    np.testing.assert_allclose(grad.cpu().numpy(), ref, rtol=RTOL, atol=ATOL)


def test_sorted_backward_accumulates_and_matches_atomic_variant():
    g = cpu_graph("powerlaw")
    out, s1, s2, _, _, _ = run_2hop("powerlaw", 15, 10, 9, dim=64, batch=256)
    go = synthetic.features(s1.size(0), 64, seed=5).cuda()
    base = synthetic.features(g.num_nodes, 64, seed=6).cuda()
    got = sorted_backward(go, s1, s2, g.num_nodes, base=base)
    want = atomic_backward(go, s1, s2, g.num_nodes, base=base)
    torch.testing.assert_close(got, want, rtol=RTOL, atol=ATOL)


def test_sorted_backward_on_c2_graph_matches_atomic_variant():
    w = synthetic.WORKLOADS["c2_2hop_powerlaw"]
    g = w.graph(0, "cuda")
    x = w.features(1, "cuda")
    fr = synthetic.root_batch(g.num_nodes, 1024, 3, device="cuda")
    _, s1, s2 = fsa.fused_sample_agg_2hop_with_samples(g.rowptr, g.col, x, fr, 15, 10, 3)
    go = synthetic.features(1024, w.dim, seed=2, device="cuda")
    got = sorted_backward(go, s1, s2, g.num_nodes)
    want = atomic_backward(go, s1, s2, g.num_nodes)
    torch.testing.assert_close(got, want, rtol=RTOL, atol=ATOL)


# ---------------------------------------------------------------------------
# Autograd behaviour of the C++ binding
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("hops", [1, 2])
def test_non_contiguous_features_give_the_same_output_and_gradient(hops):
    g = cpu_graph("powerlaw")
    rp, cl = dev_graph("powerlaw")
    base = cpu_features(g.num_nodes, 24).cuda()
    fr = frontier("powerlaw", 64, 3).cuda()
    go = synthetic.features(64, 24, seed=8).cuda()

    def run(x):
        if hops == 1:
            return fsa.fused_sample_agg(rp, cl, x, fr, 10, replay_seed=4)
        return fsa.fused_sample_agg_2hop(rp, cl, x, fr, 8, 4, replay_seed=4)

    xa = base.clone().requires_grad_(True)
    oa = run(xa)
    oa.backward(go)
    # same values, transposed storage: a non-contiguous leaf
    xb = base.t().contiguous().t().requires_grad_(True)
    assert not xb.is_contiguous()
    ob = run(xb)
    ob.backward(go)
    assert torch.equal(oa.view(torch.int32), ob.view(torch.int32))
    torch.testing.assert_close(xb.grad, xa.grad, rtol=RTOL, atol=ATOL)


def test_no_grad_mode_records_no_graph_and_allocates_no_gradient():
    rp, cl = dev_graph("powerlaw")
    g = cpu_graph("powerlaw")
    x = cpu_features(g.num_nodes, 16).cuda().requires_grad_(True)
    fr = frontier("powerlaw", 32, 1).cuda()
    torch.cuda.synchronize()
    with torch.no_grad():
        before = torch.cuda.memory_allocated()
        out = fsa.fused_sample_agg_2hop(rp, cl, x, fr, 8, 4, replay_seed=2)
        torch.cuda.synchronize()
        # ids for replay are captured (x.requires_grad), the dense N x D
        # gradient buffer is not
        assert torch.cuda.memory_allocated() - before < g.num_nodes * 16 * 4
    assert out.grad_fn is None and not out.requires_grad


def test_gradient_accumulates_over_two_backwards():
    g = cpu_graph("hub")
    rp, cl = dev_graph("hub")
    x = cpu_features(g.num_nodes, 20).cuda().requires_grad_(True)
    fr = frontier("hub", 48, 5).cuda()
    go = synthetic.features(48, 20, seed=9).cuda()
    fsa.fused_sample_agg_2hop(rp, cl, x, fr, 5, 10, replay_seed=6).backward(go)
    once = x.grad.clone()
    fsa.fused_sample_agg_2hop(rp, cl, x, fr, 5, 10, replay_seed=6).backward(go)
    torch.testing.assert_close(x.grad, 2 * once, rtol=RTOL, atol=ATOL)


# ---------------------------------------------------------------------------
# Fanouts at the shared-memory limit (f1 + f1 * f2 <= 12000)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("fan", [(5, 2399), (1, 11999), (109, 109), (5999, 1)])
def test_2hop_at_the_entry_limit_matches_oracle(fan):
    # hub graph: root 9 links to rows 0 (60,000 neighbours), 8 (20,000), 6
    # and 7 (1024 / 1025), so second-hop rows draw far past the fanout
    k1, k2 = fan
    assert k1 + k1 * k2 <= 12000
    g = cpu_graph("hub")
    out, s1, s2, ref_out, r1, r2 = run_2hop("hub", k1, k2, 3, dim=8, batch=16)
    np.testing.assert_array_equal(s1.cpu().numpy(), r1)
    np.testing.assert_array_equal(s2.cpu().numpy(), r2)
    assert_bit_equal(out, ref_out)
    go = synthetic.features(16, 8, seed=4)
    grad = atomic_backward(go.cuda(), s1, s2, g.num_nodes)
    ref = oracle.backward_2hop(go.numpy(), r1, r2, g.num_nodes)
    np.testing.assert_allclose(grad.cpu().numpy(), ref, rtol=RTOL, atol=ATOL)


def test_2hop_just_over_the_entry_limit_is_rejected():
    rp, cl = dev_graph("hub")
    x = cpu_features(70_000, 8).cuda()
    fr = frontier("hub", 16, 3).cuda()
    with pytest.raises(RuntimeError, match="shared memory"):
        fsa.fused_sample_agg_2hop(rp, cl, x, fr, 5, 2400)
