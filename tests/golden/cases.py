"""Definitions of the golden-vector cases.

The same definitions are used by make_golden.py (which runs the reference's
own CUDA op on a B200 and records its sampled ids, outputs and gradients)
and by tests/test_oracle_golden.py (which checks the CPU oracle against the
recorded vectors).  All graphs are generated on the CPU from fixed seeds, so
both sides see identical inputs; each fixture also stores the graph digest.

The reference's tests carry no golden vectors (its checks are
self-consistency only), so these fixtures are the pin for sampled-id parity.
"""

from __future__ import annotations

import torch

from fusesampleagg_b200 import synthetic

U64_MAX = (1 << 64) - 1


def toy_graph() -> synthetic.Graph:
    """8 nodes: an empty row (2), a one-neighbour row (4), rows shorter and
    longer than the fanouts used below."""
    rows = {
        0: [1, 2, 5],
        1: [0, 3],
        2: [],
        3: [0, 1, 2, 4, 6, 7],
        4: [3],
        5: [0, 6, 7],
        6: [2, 3, 5, 7],
        7: [0, 1, 3, 4, 5, 6],
    }
    rowptr = [0]
    col = []
    for r in range(8):
        col += rows[r]
        rowptr.append(len(col))
    return synthetic.Graph(torch.tensor(rowptr, dtype=torch.int32),
                           torch.tensor(col, dtype=torch.int32))


def hub_graph() -> synthetic.Graph:
    """Rows around every reservoir boundary plus very long rows.

    Row 0 has 60,000 neighbours, row 8 has 20,000, rows 2..7 have degree
    10, 11, 9, 1, 1024, 1025 and row 1 is empty; row 9 links to the hubs so
    they appear as second-hop rows; the remaining rows are short random rows.
    """
    n = 70_000
    g = torch.Generator().manual_seed(7)
    srcs = [torch.zeros(60_000, dtype=torch.int64)]
    dsts = [torch.arange(1, 60_001)]
    for r, d in ((2, 10), (3, 11), (4, 9), (5, 1), (6, 1024), (7, 1025), (8, 20_000)):
        srcs.append(torch.full((d,), r, dtype=torch.int64))
        dsts.append(torch.randperm(n - 10, generator=g)[:d] + 10)
    srcs.append(torch.full((5,), 9, dtype=torch.int64))
    dsts.append(torch.tensor([0, 3, 6, 7, 8]))
    deg = torch.randint(0, 8, (n - 10,), generator=g)
    srcs.append(torch.repeat_interleave(torch.arange(10, n), deg))
    dsts.append(torch.randint(0, n, (int(deg.sum()),), generator=g))
    return synthetic.csr_from_edges(torch.cat(srcs), torch.cat(dsts), n)


def uniform_graph() -> synthetic.Graph:
    """The 1-hop benchmark shape: N=10k, Poisson(10) out-degree, 2% empty."""
    return synthetic.poisson_graph(10_000, 10.0, 0.02, seed=0, device="cpu")


def powerlaw_graph() -> synthetic.Graph:
    """A small Chung-Lu graph (N=20k, ~600k edges, exponent 2.1, cap 5000)."""
    return synthetic.chung_lu_graph(20_000, 600_000, 2.1, 5_000, seed=0, device="cpu")


GRAPHS = {
    "toy": toy_graph,
    "hub": hub_graph,
    "uniform": uniform_graph,
    "powerlaw": powerlaw_graph,
}


def frontier_for(graph_name: str, graph: synthetic.Graph, batch: int, seed: int) -> torch.Tensor:
    """Roots of a case; ``seed == -1`` selects the ``batch`` highest-degree
    nodes (hub roots: every first-hop row is long)."""
    if seed == -1:
        order = torch.sort(graph.degrees(), descending=True, stable=True).indices
        return order[:batch].to(torch.int32)
    if graph_name == "toy":
        # Every node, the empty row included, and a repeated root.
        return torch.tensor([0, 3, 2, 6, 7, 1, 4, 5, 3], dtype=torch.int32)
    if graph_name == "hub":
        head = torch.arange(0, 10, dtype=torch.int32)
        rest = synthetic.root_batch(graph.num_nodes - 10, max(batch - 10, 0), seed) + 10
        return torch.cat([head, rest.to(torch.int32)])
    return synthetic.root_batch(graph.num_nodes, batch, seed)


def _c(name, graph, hops, fanouts, seed, dim, batch=0, root_seed=0, grad=False, store_out=False):
    return dict(name=name, graph=graph, hops=hops, fanouts=tuple(fanouts), seed=seed, dim=dim,
                batch=batch, root_seed=root_seed, grad=grad, store_out=store_out)


CASES = [
    # toy graph: every fanout boundary, narrow and odd widths, gradients.
    *[_c(f"toy_1hop_k{k}_d{d}", "toy", 1, (k,), 17, d, grad=True, store_out=True)
      for k in (1, 2, 3, 5) for d in (1, 5, 33)],
    *[_c(f"toy_2hop_{a}x{b}_d{d}", "toy", 2, (a, b), s, d, grad=True, store_out=True)
      for (a, b, s) in ((3, 2, 7), (2, 3, 1234), (5, 4, 0), (1, 1, U64_MAX)) for d in (1, 19)],
    # hub graph: long rows split across many threads.
    *[_c(f"hub_1hop_k{k}_s{s}", "hub", 1, (k,), s, 8, batch=64, root_seed=3)
      for k in (1, 10, 11, 1024) for s in (0, 99)],
    *[_c(f"hub_2hop_{a}x{b}_s{s}", "hub", 2, (a, b), s, 8, batch=48, root_seed=4)
      for (a, b) in ((5, 10), (15, 10)) for s in (5, U64_MAX)],
    # the 1-hop benchmark graph and batch (fanout 10, seed 0).
    _c("uniform_1hop_k10_b1024", "uniform", 1, (10,), 0, 128, batch=1024, root_seed=0),
    # power law: the 2-hop benchmark fanouts and the KG/wide fanouts.
    _c("powerlaw_2hop_15x10_s0", "powerlaw", 2, (15, 10), 0, 100, batch=256, root_seed=0),
    _c("powerlaw_2hop_15x10_s1", "powerlaw", 2, (15, 10), 1, 100, batch=128, root_seed=1),
    _c("powerlaw_2hop_25x10_s3", "powerlaw", 2, (25, 10), 3, 33, batch=96, root_seed=2),
    _c("powerlaw_2hop_8x4_s9", "powerlaw", 2, (8, 4), 9, 64, batch=256, root_seed=3),
    _c("powerlaw_1hop_k8_s1234", "powerlaw", 1, (8,), 1234, 100, batch=256, root_seed=4),
    _c("powerlaw_1hop_k100_s2", "powerlaw", 1, (100,), 2, 3, batch=128, root_seed=5),
    # hub roots: long first-hop rows for every root
    _c("powerlaw_2hop_15x10_hubroots", "powerlaw", 2, (15, 10), 11, 16, batch=128, root_seed=-1),
    _c("powerlaw_1hop_k10_hubroots", "powerlaw", 1, (10,), 12, 16, batch=128, root_seed=-1),
]


def features_for(case: dict, num_nodes: int) -> torch.Tensor:
    return synthetic.features(num_nodes, case["dim"], seed=1, device="cpu")


def grad_out_for(case: dict, batch: int) -> torch.Tensor:
    return synthetic.features(batch, case["dim"], seed=2, device="cpu")
