"""Owner-computes row-sharded 2-hop backward through the C ABI on one GPU:
W shards and W exchange regions on the same device stand in for W ranks
(fsa_sharded_publish_2hop per rank, then fsa_sample_agg_2hop_backward_sharded_pull
per shard).  The concatenated gradient shards must equal the unsharded
backward of all ranks' roots (rtol 1e-5 / atol 1e-6: the additions land in
a different order).  The two-process run over NVLink is in
tests/test_sharded_gpu.py.
"""

from __future__ import annotations

import ctypes
import functools

import pytest
import torch

from fusesampleagg_b200 import _lib, synthetic
from tests.golden import cases as C

pytestmark = pytest.mark.gpu
L = _lib.LIB
RTOL, ATOL = 1e-5, 1e-6


@functools.lru_cache(maxsize=None)
def graph(name):
    g = C.GRAPHS[name]()
    return g, g.rowptr.cuda(), g.col.cuda()


def stream():
    return torch.cuda.current_stream().cuda_stream


def sample(name, dim, k1, k2, batch, seed, offset):
    g, rp, cl = graph(name)
    x = synthetic.features(g.num_nodes, dim, seed=1, device="cuda")
    fr = synthetic.root_batch(g.num_nodes, batch, seed=seed, device="cuda")
    out = torch.empty(batch, dim, device="cuda")
    s1 = torch.empty(batch, k1, dtype=torch.int32, device="cuda")
    s2 = torch.empty(batch, k1, k2, dtype=torch.int32, device="cuda")
    ws_bytes = L.fsa_sample_agg_2hop_workspace_size(batch, k1, k2, 1, 1)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    if batch > 0:
        _lib.check(L.fsa_sample_agg_2hop_forward(
            rp.data_ptr(), cl.data_ptr(), g.num_nodes, cl.numel(), x.data_ptr(), dim,
            fr.data_ptr(), batch, offset, k1, k2, seed, out.data_ptr(), s1.data_ptr(),
            s2.data_ptr(), ws.data_ptr(), ws_bytes, None, 0, stream()), "forward")
    return s1, s2


def run(name, dim, k1, k2, batches, world):
    g, _, _ = graph(name)
    n = g.num_nodes
    rows = -(-n // world)
    ranks = []
    for r, batch in enumerate(batches):
        s1, s2 = sample(name, dim, k1, k2, batch, 40 + r, sum(batches[:r]))
        go = synthetic.features(batch, dim, seed=7 + r, device="cuda")
        ranks.append((s1, s2, go))
    need = max(L.fsa_exchange_bytes(b, k1, k2, dim) for b in batches)
    regions = [torch.full((need,), 0xAB, dtype=torch.uint8, device="cuda") for _ in range(world)]
    for (s1, s2, go), reg, b in zip(ranks, regions, batches):
        _lib.check(L.fsa_sharded_publish_2hop(reg.data_ptr(), need, go.data_ptr(), s1.data_ptr(),
                                              s2.data_ptr(), b, dim, k1, k2, stream()), "publish")
    ptrs = (ctypes.c_void_p * world)(*[r.data_ptr() for r in regions])
    shards = torch.zeros(world * rows, dim, device="cuda")
    for r in range(world):
        _lib.check(L.fsa_sample_agg_2hop_backward_sharded_pull(
            ptrs, need, world, r, shards[r * rows].data_ptr(), rows, n, dim, k1, k2, None, 0,
            stream()),
            "pull")
    want = torch.zeros(n, dim, device="cuda")
    for (s1, s2, go), b in zip(ranks, batches):
        _lib.check(L.fsa_sample_agg_2hop_backward(go.data_ptr(), s1.data_ptr(), s2.data_ptr(), b,
                                                  dim, k1, k2, want.data_ptr(), n, stream()),
                   "backward")
    torch.cuda.synchronize()
    return shards[:n], want


@pytest.mark.parametrize("name,dim,k1,k2,batches", [
    ("powerlaw", 100, 15, 10, (256, 256)),
    ("powerlaw", 64, 15, 10, (100, 101, 99, 0, 64, 1, 5, 200)),
    ("powerlaw", 33, 8, 4, (128, 127, 128)),
    ("powerlaw", 6, 25, 10, (64, 64, 64, 64)),
    ("hub", 8, 40, 20, (48, 47)),
    ("hub", 16, 5, 400, (48, 47)),      # records over a warp's slice: a CTA per unit
    ("hub", 8, 5, 2399, (16, 16, 16)),  # records over 16 KB: ids staged, gradient read in place
    ("toy", 4, 3, 2, (6, 0)),
])
def test_pull_backward_matches_unsharded(name, dim, k1, k2, batches):
    world = len(batches)
    got, want = run(name, dim, k1, k2, batches, world)
    torch.testing.assert_close(got, want, rtol=RTOL, atol=ATOL)
    assert _lib.device_status(torch.cuda.current_device(), reset=True) == 0


def test_one_shard_of_all_rows_sums_every_rank():
    """The replicated-feature exchange (GradientExchange): each rank pulls
    with one shard covering all N rows, so its gradient is the sum over all
    ranks' roots -- the all-reduced gradient."""
    name, dim, k1, k2, batches = "powerlaw", 64, 15, 10, (128, 128, 128)
    g, _, _ = graph(name)
    n = g.num_nodes
    world = len(batches)
    ranks = []
    for r, batch in enumerate(batches):
        s1, s2 = sample(name, dim, k1, k2, batch, 60 + r, r * batch)
        ranks.append((s1, s2, synthetic.features(batch, dim, seed=9 + r, device="cuda")))
    need = L.fsa_exchange_bytes(max(batches), k1, k2, dim)
    regions = [torch.empty((need,), dtype=torch.uint8, device="cuda") for _ in range(world)]
    for (s1, s2, go), reg, b in zip(ranks, regions, batches):
        _lib.check(L.fsa_sharded_publish_2hop(reg.data_ptr(), need, go.data_ptr(), s1.data_ptr(),
                                              s2.data_ptr(), b, dim, k1, k2, stream()), "publish")
    ptrs = (ctypes.c_void_p * world)(*[r.data_ptr() for r in regions])
    got = torch.zeros(n, dim, device="cuda")
    _lib.check(L.fsa_sample_agg_2hop_backward_sharded_pull(
        ptrs, need, world, 0, got.data_ptr(), n, n, dim, k1, k2, None, 0, stream()), "pull")
    want = torch.zeros(n, dim, device="cuda")
    for (s1, s2, go), b in zip(ranks, batches):
        _lib.check(L.fsa_sample_agg_2hop_backward(go.data_ptr(), s1.data_ptr(), s2.data_ptr(), b,
                                                  dim, k1, k2, want.data_ptr(), n, stream()),
                   "backward")
    torch.cuda.synchronize()
    torch.testing.assert_close(got, want, rtol=RTOL, atol=ATOL)


def test_pull_lists_the_rows_it_touched():
    """With a touched-row list the pull call also writes, per (region, root)
    unit, the local row of every owned id (-1 for the others and for units
    past a region's root count): the rows a persistent shard clears next."""
    name, dim, k1, k2, batches = "powerlaw", 16, 8, 4, (64, 50, 64)
    g, _, _ = graph(name)
    n = g.num_nodes
    world = len(batches)
    rows = -(-n // world)
    ranks = []
    for r, batch in enumerate(batches):
        s1, s2 = sample(name, dim, k1, k2, batch, 80 + r, r * 64)
        ranks.append((s1, s2, synthetic.features(batch, dim, seed=3 + r, device="cuda")))
    need = L.fsa_exchange_bytes(max(batches), k1, k2, dim)
    regions = [torch.empty((need,), dtype=torch.uint8, device="cuda") for _ in range(world)]
    for (s1, s2, go), reg, b in zip(ranks, regions, batches):
        _lib.check(L.fsa_sharded_publish_2hop(reg.data_ptr(), need, go.data_ptr(), s1.data_ptr(),
                                              s2.data_ptr(), b, dim, k1, k2, stream()), "publish")
    ptrs = (ctypes.c_void_p * world)(*[r.data_ptr() for r in regions])
    cap = (need - 256) // (L.fsa_exchange_bytes(1, k1, k2, dim) - 256)
    shard = 1
    touched = torch.full((cap * world * k1 * k2,), 12345, dtype=torch.int32, device="cuda")
    grad = torch.zeros(rows, dim, device="cuda")
    _lib.check(L.fsa_sample_agg_2hop_backward_sharded_pull(
        ptrs, need, world, shard, grad.data_ptr(), rows, n, dim, k1, k2, touched.data_ptr(),
        touched.numel(), stream()), "pull")
    torch.cuda.synchronize()
    got = touched.cpu().view(cap, world, k1 * k2)
    lo = shard * rows
    for s, (s1, s2, _) in enumerate(ranks):
        ids = s2.cpu().view(-1, k1 * k2)
        want = torch.where((ids >= lo) & (ids < lo + rows) & (ids < n), ids - lo,
                           torch.full_like(ids, -1))
        assert torch.equal(got[:ids.size(0), s], want)
        assert bool((got[ids.size(0):, s] == -1).all())
    # the listed rows are exactly the rows the call added into
    listed = got[got >= 0].unique()
    nonzero = (grad.cpu().abs().sum(1) > 0).nonzero().flatten().to(torch.int32)
    assert set(nonzero.tolist()) <= set(listed.tolist())
