"""CSR preparation on the GPU, in the reference's on-disk format.

The reference prepares graphs on the host with numpy (an incoming-edge CSR:
row = edge target, neighbours = sources sorted ascending within a row,
`scripts/download_data.py:10-22`; KG graphs add the reversed triples,
`scripts/kg_prepare_csr.py:76-83`) and stores ``rowptr`` / ``col`` as int32
arrays in ``csr_adj.npz`` (`scripts/download_data.py:25-30`).  This module
builds the same arrays on the GPU — one int64 sort of (row, neighbour) keys,
a histogram and a prefix sum, with every offset in int64 so that graphs up
to 2^31 - 1 edges (the 100M-node / 1.6B-edge configuration) build without
overflow — and reads and writes the same file format.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

INT32_MAX = 2**31 - 1


def build_csr(rows: torch.Tensor, neighbors: torch.Tensor, num_nodes: int,
              device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """int32 (rowptr[num_nodes + 1], col[E]) with row r listing the
    `neighbors` of the edges whose `rows` entry is r, ascending; duplicate
    edges are kept (as the reference's builders keep them).

    `rows` / `neighbors` are integer tensors of equal length (any device;
    the work runs on `device`, default: theirs)."""
    if rows.shape != neighbors.shape or rows.dim() != 1:
        raise ValueError("rows and neighbors must be 1-D tensors of equal length")
    num_nodes = int(num_nodes)
    if num_nodes < 0 or num_nodes > INT32_MAX:
        raise ValueError("num_nodes must be in [0, 2^31 - 1]")
    if rows.numel() > INT32_MAX:
        raise ValueError("edge count does not fit int32 CSR offsets")
    dev = torch.device(device) if device is not None else rows.device
    r = rows.to(dev, torch.int64)
    c = neighbors.to(dev, torch.int64)
    if r.numel() and (int(r.min()) < 0 or int(r.max()) >= num_nodes
                      or int(c.min()) < 0 or int(c.max()) >= num_nodes):
        raise ValueError("edge endpoints must be in [0, num_nodes)")
    key = r * num_nodes + c          # < 2^62 for num_nodes < 2^31
    del r
    key = torch.sort(key).values
    row_of = torch.div(key, num_nodes, rounding_mode="floor") if num_nodes else key
    col = (key - row_of * num_nodes).to(torch.int32)
    counts = torch.bincount(row_of, minlength=num_nodes)
    del key, row_of
    rowptr = torch.zeros(num_nodes + 1, dtype=torch.int64, device=dev)
    torch.cumsum(counts, 0, out=rowptr[1:])
    return rowptr.to(torch.int32), col


def incoming_csr(edge_index: torch.Tensor, num_nodes: int, device=None):
    """The reference's `edge_index_to_incoming_csr`: row = target
    (edge_index[1]), neighbours = sources (edge_index[0])."""
    if edge_index.dim() != 2 or edge_index.size(0) != 2:
        raise ValueError("edge_index must be [2, E]")
    return build_csr(edge_index[1], edge_index[0], num_nodes, device)


def kg_csr(heads: torch.Tensor, tails: torch.Tensor, num_nodes: int, undirected: bool = True,
           device=None):
    """The reference's KG adjacency: head -> tail rows, plus tail -> head
    when `undirected`."""
    rows, nbrs = heads, tails
    if undirected:
        rows = torch.cat([heads, tails])
        nbrs = torch.cat([tails, heads])
    return build_csr(rows, nbrs, num_nodes, device)


def save_csr(path, rowptr: torch.Tensor, col: torch.Tensor) -> Path:
    """Writes ``csr_adj.npz`` (compressed, int32 ``rowptr`` and ``col``) into
    `path` (a directory) or to `path` itself when it ends in ``.npz``."""
    p = Path(path)
    if p.suffix != ".npz":
        p.mkdir(parents=True, exist_ok=True)
        p = p / "csr_adj.npz"
    np.savez_compressed(p, rowptr=rowptr.cpu().numpy().astype(np.int32, copy=False),
                        col=col.cpu().numpy().astype(np.int32, copy=False))
    return p


def load_csr(path, device="cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """Reads ``csr_adj.npz`` (a directory holding it, or the file) and
    checks the CSR invariants the operator relies on."""
    p = Path(path)
    if p.is_dir():
        p = p / "csr_adj.npz"
    with np.load(p) as z:
        rowptr = torch.from_numpy(np.ascontiguousarray(z["rowptr"], dtype=np.int32))
        col = torch.from_numpy(np.ascontiguousarray(z["col"], dtype=np.int32))
    if rowptr.numel() < 1 or int(rowptr[0]) != 0 or int(rowptr[-1]) != col.numel():
        raise ValueError(f"{p}: rowptr must start at 0 and end at len(col)")
    if rowptr.numel() > 1 and bool((rowptr[1:] < rowptr[:-1]).any()):
        raise ValueError(f"{p}: rowptr must be non-decreasing")
    return rowptr.to(device), col.to(device)
