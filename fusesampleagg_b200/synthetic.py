"""Seeded synthetic CSR graphs, features and root batches for the benchmark
workloads and the tests.

CSR convention (the reference's data preparation,
scripts/download_data.py:10-22 and scripts/kg_prepare_csr.py:11-23):
``rowptr`` int32[N+1], ``col`` int32[E], neighbours sorted ascending within
each row, no duplicate (row, neighbour) pairs.  Sampled ids depend on the
in-row order, so every generator here sorts.

Every generator is a pure function of its arguments (a ``torch.Generator``
seeded from ``seed`` on the requested device), so two processes with the same
torch build produce identical graphs.  CPU and CUDA generators produce
different streams; the tests only compare graphs generated on the same kind
of device.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import torch


@dataclass
class Graph:
    rowptr: torch.Tensor  # int32 [N+1]
    col: torch.Tensor  # int32 [E]

    @property
    def num_nodes(self) -> int:
        return int(self.rowptr.numel()) - 1

    @property
    def num_edges(self) -> int:
        return int(self.col.numel())

    def degrees(self) -> torch.Tensor:
        return (self.rowptr[1:] - self.rowptr[:-1]).to(torch.int64)

    def to(self, device) -> "Graph":
        return Graph(self.rowptr.to(device), self.col.to(device))

    def digest(self) -> str:
        """SHA-256 of the CSR arrays (little-endian int32)."""
        h = hashlib.sha256()
        h.update(self.rowptr.cpu().numpy().tobytes())
        h.update(self.col.cpu().numpy().tobytes())
        return h.hexdigest()


# Each generator mixes its purpose into the seed, so that e.g. graph seed 0
# and root-batch seed 0 do not share a random stream (they would otherwise
# draw the same permutation, making root batch 0 the graph's top hubs).
_SALT = {"graph": 0x6772617068, "poisson": 0x706F6973, "features": 0x66656174,
         "roots": 0x726F6F7473}


def _generator(seed: int, device, purpose: str) -> torch.Generator:
    v = (int(seed) * 0x9E3779B97F4A7C15 + _SALT[purpose]) & ((1 << 64) - 1)
    v ^= v >> 31
    v = (v * 0xBF58476D1CE4E5B9) & ((1 << 64) - 1)
    v ^= v >> 29
    return torch.Generator(device=torch.device(device)).manual_seed(v & ((1 << 63) - 1))


def csr_from_edges(src: torch.Tensor, dst: torch.Tensor, num_nodes: int,
                   max_degree: int | None = None) -> Graph:
    """Builds a deduplicated CSR sorted within rows from directed edges.

    Rows longer than ``max_degree`` keep their ``max_degree`` smallest
    neighbour ids (node ids are randomly permuted by the generators, so this
    is a uniform subset of the row).
    """
    device = src.device
    key = src.to(torch.int64) * num_nodes + dst.to(torch.int64)
    key = torch.sort(key).values
    key = torch.unique_consecutive(key)
    rows = torch.div(key, num_nodes, rounding_mode="floor")
    cols = key - rows * num_nodes
    del key
    counts = torch.bincount(rows, minlength=num_nodes)
    if max_degree is not None and int(counts.max()) > max_degree:
        starts = torch.zeros(num_nodes + 1, dtype=torch.int64, device=device)
        torch.cumsum(counts, 0, out=starts[1:])
        pos = torch.arange(rows.numel(), device=device) - starts[rows]
        keep = pos < max_degree
        rows = rows[keep]
        cols = cols[keep]
        counts = torch.bincount(rows, minlength=num_nodes)
    rowptr = torch.zeros(num_nodes + 1, dtype=torch.int64, device=device)
    torch.cumsum(counts, 0, out=rowptr[1:])
    if int(rowptr[-1]) >= 2**31:
        raise ValueError("edge count does not fit int32 CSR offsets")
    return Graph(rowptr.to(torch.int32), cols.to(torch.int32))


def poisson_graph(num_nodes: int, mean_degree: float, zero_fraction: float,
                  seed: int, device="cpu") -> Graph:
    """Uniform random directed graph: out-degree ~ Poisson(mean_degree),
    self-loops excluded, ``zero_fraction`` of the nodes forced to degree 0."""
    g = _generator(seed, device, "poisson")
    deg = torch.poisson(torch.full((num_nodes,), float(mean_degree), device=device),
                        generator=g).to(torch.int64)
    n_zero = int(round(zero_fraction * num_nodes))
    if n_zero:
        zero = torch.randperm(num_nodes, generator=g, device=device)[:n_zero]
        deg[zero] = 0
    src = torch.repeat_interleave(torch.arange(num_nodes, device=device), deg)
    # dst = src + U{1..N-1} (mod N) is uniform over the other N-1 nodes.
    shift = torch.randint(1, max(num_nodes, 2), (src.numel(),), generator=g, device=device)
    dst = (src + shift) % num_nodes
    return csr_from_edges(src, dst, num_nodes)


def chung_lu_weights(num_nodes: int, num_edges: int, exponent: float,
                     max_degree: int, device="cpu") -> torch.Tensor:
    """Expected degrees w_i = c * (i+1)^(-1/(exponent-1)) capped at max_degree,
    with c chosen so that sum(w) = num_edges (directed)."""
    alpha = 1.0 / (exponent - 1.0)
    base = torch.arange(1, num_nodes + 1, dtype=torch.float64, device=device).pow(-alpha)
    lo, hi = 0.0, float(num_edges) * 4.0
    for _ in range(200):
        mid = 0.5 * (lo + hi)
        if float(torch.clamp(base * mid, max=max_degree).sum()) < num_edges:
            lo = mid
        else:
            hi = mid
    return torch.clamp(base * hi, max=max_degree)


def chung_lu_graph(num_nodes: int, num_edges: int, exponent: float,
                   max_degree: int, seed: int, device="cpu",
                   oversample: float = 1.0, chunk: int = 1 << 26) -> Graph:
    """Symmetric Chung-Lu power-law graph.

    ``num_edges * oversample / 2`` undirected pairs are drawn with both ends
    ~ w (inverse CDF), self-loops dropped, both directions added, duplicates
    removed, rows capped at ``max_degree``, and node ids randomly permuted so
    that hubs are scattered over the id space.  ``oversample`` compensates
    for the duplicate pairs that hubs produce.
    """
    g = _generator(seed, device, "graph")
    w = chung_lu_weights(num_nodes, num_edges, exponent, max_degree, device)
    # The float64 prefix sum runs on the host: a GPU scan's association
    # order can vary from run to run, which moved a few sampled endpoints
    # across bin edges and gave ranks of one job slightly different graphs.
    cdf = torch.cumsum(w.cpu(), 0).to(w.device)
    total = float(cdf[-1])
    perm = torch.randperm(num_nodes, generator=g, device=device).to(torch.int32)
    pairs = int(num_edges * oversample) // 2
    srcs, dsts = [], []
    for start in range(0, pairs, chunk):
        m = min(chunk, pairs - start)
        u = torch.searchsorted(cdf, torch.rand(m, dtype=torch.float64, generator=g, device=device) * total)
        v = torch.searchsorted(cdf, torch.rand(m, dtype=torch.float64, generator=g, device=device) * total)
        u.clamp_(max=num_nodes - 1)
        v.clamp_(max=num_nodes - 1)
        keep = u != v
        u = perm[u[keep]]
        v = perm[v[keep]]
        srcs += [u, v]
        dsts += [v, u]
    src = torch.cat(srcs)
    dst = torch.cat(dsts)
    del srcs, dsts
    return csr_from_edges(src, dst, num_nodes, max_degree=max_degree)


def features(num_nodes: int, dim: int, seed: int, device="cpu", std: float = 1.0) -> torch.Tensor:
    g = _generator(seed, device, "features")
    x = torch.randn(num_nodes, dim, generator=g, device=device, dtype=torch.float32)
    if std != 1.0:
        x.mul_(std)
    return x


def root_batch(num_nodes: int, batch: int, seed: int, device="cpu") -> torch.Tensor:
    """``batch`` distinct uniformly drawn root ids (int32)."""
    g = _generator(seed, device, "roots")
    if batch > num_nodes:
        raise ValueError("batch larger than the node count")
    if num_nodes <= 1 << 22:
        return torch.randperm(num_nodes, generator=g, device=device)[:batch].to(torch.int32)
    # Large N: draw with replacement, keep first occurrences, top up.
    picked = torch.empty(0, dtype=torch.int64, device=device)
    while picked.numel() < batch:
        cand = torch.randint(0, num_nodes, (2 * batch,), generator=g, device=device)
        picked = torch.cat([picked, cand])
        uniq, inv = torch.unique(picked, return_inverse=True)
        first = torch.full((uniq.numel(),), picked.numel(), dtype=torch.int64, device=device)
        first.scatter_reduce_(0, inv, torch.arange(picked.numel(), device=device), "amin")
        picked = picked[torch.sort(first).values]
    return picked[:batch].to(torch.int32)


# ---------------------------------------------------------------------------
# Named workloads (sizes of the benchmark configurations)
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class Workload:
    name: str
    hops: int
    fanouts: tuple
    num_nodes: int
    num_edges: int
    dim: int
    batch: int
    kind: str  # "poisson" or "chung_lu"
    exponent: float = 0.0
    max_degree: int = 0
    mean_degree: float = 0.0
    zero_fraction: float = 0.0
    oversample: float = 1.0
    feature_std: float = 1.0

    def describe(self) -> dict:
        return {
            "workload": self.name,
            "hops": self.hops,
            "fanouts": list(self.fanouts),
            "num_nodes": self.num_nodes,
            "target_edges": self.num_edges,
            "feature_dim": self.dim,
            "roots_per_batch": self.batch,
            "graph": self.kind,
            "exponent": self.exponent or None,
            "max_degree_cap": self.max_degree or None,
        }

    def graph(self, seed: int = 0, device="cpu") -> Graph:
        if self.kind == "poisson":
            return poisson_graph(self.num_nodes, self.mean_degree, self.zero_fraction, seed, device)
        return chung_lu_graph(self.num_nodes, self.num_edges, self.exponent, self.max_degree,
                              seed, device, oversample=self.oversample)

    def features(self, seed: int = 1, device="cpu") -> torch.Tensor:
        return features(self.num_nodes, self.dim, seed, device, std=self.feature_std)


WORKLOADS = {
    # 1-hop, fanout 10, uniform Poisson(10) graph with 2% empty rows.
    "c1_1hop_uniform": Workload("c1_1hop_uniform", 1, (10,), 10_000, 100_000, 128, 1024,
                                "poisson", mean_degree=10.0, zero_fraction=0.02),
    # 2-hop (15,10), Chung-Lu power law N=2.45M, ~123M directed edges, D=100.
    "c2_2hop_powerlaw": Workload("c2_2hop_powerlaw", 2, (15, 10), 2_450_000, 123_000_000, 100,
                                 1024, "chung_lu", exponent=2.1, max_degree=20_000,
                                 oversample=1.03),
    # Wide features: 2-hop (25,10), N=233k, ~114M edges, exponent 1.9, D=602.
    "c3_2hop_wide": Workload("c3_2hop_wide", 2, (25, 10), 233_000, 114_000_000, 602, 1024,
                             "chung_lu", exponent=1.9, max_degree=10_700, oversample=1.0),
    # Knowledge-graph encoder shapes (512 heads): (a) 94k entities D=200, (b) 2.5M D=100.
    "c4a_kg_2hop": Workload("c4a_kg_2hop", 2, (8, 4), 94_000, 10_200_000, 200, 512,
                            "chung_lu", exponent=2.0, max_degree=93_999, feature_std=0.1),
    "c4a_kg_1hop": Workload("c4a_kg_1hop", 1, (8,), 94_000, 10_200_000, 200, 512,
                            "chung_lu", exponent=2.0, max_degree=93_999, feature_std=0.1),
    "c4b_kg_2hop": Workload("c4b_kg_2hop", 2, (8, 4), 2_500_000, 32_000_000, 100, 512,
                            "chung_lu", exponent=2.2, max_degree=2_499_999, feature_std=0.1),
    # Multi-GPU scale: N=100M, 1.6B edges, D=128, 65,536 roots per GPU.
    "c5_2hop_100m": Workload("c5_2hop_100m", 2, (15, 10), 100_000_000, 1_600_000_000, 128,
                             65_536, "chung_lu", exponent=2.1, max_degree=20_000),
}


def degree_stats(graph: Graph) -> dict:
    deg = graph.degrees()
    n = max(graph.num_nodes, 1)
    e = max(graph.num_edges, 1)
    deg_f = deg.to(torch.float64)
    return {
        "num_nodes": graph.num_nodes,
        "num_edges": graph.num_edges,
        "mean_degree": graph.num_edges / n,
        "max_degree": int(deg.max()) if deg.numel() else 0,
        "size_biased_mean_degree": float((deg_f * deg_f).sum() / e),
        "frac_degree_lt_10": float((deg < 10).to(torch.float64).mean()) if deg.numel() else 0.0,
        "frac_degree_0": float((deg == 0).to(torch.float64).mean()) if deg.numel() else 0.0,
    }

