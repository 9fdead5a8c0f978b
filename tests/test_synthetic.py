"""Synthetic workload generators: CSR invariants (int32, sorted within rows,
no duplicates), degree caps, empty-row fraction, distinct roots, and
determinism of the seeded streams."""

from __future__ import annotations

import pytest
import torch

from fusesampleagg_b200 import synthetic


def check_csr(g: synthetic.Graph, self_loops_allowed=True):
    assert g.rowptr.dtype == torch.int32 and g.col.dtype == torch.int32
    assert int(g.rowptr[0]) == 0 and int(g.rowptr[-1]) == g.num_edges
    deg = g.degrees()
    assert bool((deg >= 0).all())
    rows = torch.repeat_interleave(torch.arange(g.num_nodes), deg)
    key = rows * g.num_nodes + g.col.long()
    assert bool((key[1:] > key[:-1]).all()), "rows must be sorted and duplicate-free"
    assert bool((g.col >= 0).all()) and bool((g.col < g.num_nodes).all())
    if not self_loops_allowed:
        assert not bool((rows == g.col.long()).any())


def test_poisson_graph_shape():
    g = synthetic.poisson_graph(10_000, 10.0, 0.02, seed=0)
    check_csr(g, self_loops_allowed=False)
    stats = synthetic.degree_stats(g)
    assert abs(stats["mean_degree"] - 10.0) < 0.5
    assert stats["frac_degree_0"] >= 0.02


def test_chung_lu_graph_shape_and_cap():
    g = synthetic.chung_lu_graph(20_000, 600_000, 2.1, 5_000, seed=0)
    check_csr(g, self_loops_allowed=False)
    stats = synthetic.degree_stats(g)
    assert stats["max_degree"] <= 5_000
    assert stats["size_biased_mean_degree"] > 5 * stats["mean_degree"]
    # symmetric: the transpose has the same edge set
    rows = torch.repeat_interleave(torch.arange(g.num_nodes), g.degrees())
    fwd = torch.sort(rows * g.num_nodes + g.col.long()).values
    bwd = torch.sort(g.col.long() * g.num_nodes + rows).values
    assert torch.equal(fwd, bwd)


def test_chung_lu_cap_truncation_keeps_csr_valid():
    g = synthetic.chung_lu_graph(3_000, 200_000, 1.9, 300, seed=1)
    check_csr(g)
    assert int(g.degrees().max()) <= 300


def test_generators_are_deterministic():
    a = synthetic.chung_lu_graph(5_000, 50_000, 2.1, 1_000, seed=3)
    b = synthetic.chung_lu_graph(5_000, 50_000, 2.1, 1_000, seed=3)
    assert a.digest() == b.digest()
    c = synthetic.chung_lu_graph(5_000, 50_000, 2.1, 1_000, seed=4)
    assert a.digest() != c.digest()


@pytest.mark.parametrize("n,b", [(100, 100), (10_000, 1024), ((1 << 22) + 5, 4096)])
def test_root_batch_distinct(n, b):
    r = synthetic.root_batch(n, b, seed=7)
    assert r.dtype == torch.int32 and r.numel() == b
    assert torch.unique(r).numel() == b
    assert int(r.min()) >= 0 and int(r.max()) < n
    assert torch.equal(r, synthetic.root_batch(n, b, seed=7))


def test_root_batch_too_large():
    with pytest.raises(ValueError):
        synthetic.root_batch(10, 11, seed=0)


def test_workload_table():
    w = synthetic.WORKLOADS["c2_2hop_powerlaw"]
    assert (w.num_nodes, w.dim, w.fanouts, w.batch) == (2_450_000, 100, (15, 10), 1024)
    assert synthetic.WORKLOADS["c1_1hop_uniform"].fanouts == (10,)
    assert synthetic.WORKLOADS["c5_2hop_100m"].batch == 65_536


def test_root_batches_are_not_degree_biased():
    """Root batches and graphs use separate random streams: the mean degree
    of a uniform root batch matches the graph's mean degree (a shared stream
    once made root batch 0 the graph's 1024 largest hubs)."""
    g = synthetic.chung_lu_graph(50_000, 1_000_000, 2.1, 5_000, seed=0)
    deg = g.degrees().to(torch.float64)
    for seed in (0, 1, 2):
        r = synthetic.root_batch(g.num_nodes, 2_000, seed=seed).long()
        assert float(deg[r].mean()) < 2.0 * float(deg.mean())
