"""CSR preparation (fusesampleagg_b200/csr.py) against a numpy restatement
of the reference's builders (scripts/download_data.py:10-22,
scripts/kg_prepare_csr.py:11-23: lexsort by (row, neighbour), bincount,
cumsum, duplicates kept), the npz round trip, and the bounds checks.  Runs on
the CPU; the same torch code runs on the GPU."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fusesampleagg_b200 import csr


def numpy_csr(num_nodes, rows, neighbors):
    order = np.lexsort((neighbors, rows))
    counts = np.bincount(rows[order], minlength=num_nodes)
    rowptr = np.zeros(num_nodes + 1, dtype=np.int64)
    np.cumsum(counts, out=rowptr[1:])
    return rowptr.astype(np.int32), neighbors[order].astype(np.int32)


@pytest.mark.parametrize("n,e,seed", [(1, 0, 0), (7, 30, 1), (1000, 20_000, 2),
                                      (50_000, 300_000, 3)])
def test_build_matches_numpy_restatement(n, e, seed):
    g = np.random.default_rng(seed)
    rows = g.integers(0, n, e)
    nbrs = g.integers(0, n, e)
    rp, col = csr.build_csr(torch.from_numpy(rows), torch.from_numpy(nbrs), n)
    ref_rp, ref_col = numpy_csr(n, rows, nbrs)
    assert rp.dtype == torch.int32 and col.dtype == torch.int32
    np.testing.assert_array_equal(rp.numpy(), ref_rp)
    np.testing.assert_array_equal(col.numpy(), ref_col)


def test_incoming_and_kg_layouts():
    g = np.random.default_rng(4)
    n = 300
    ei = torch.from_numpy(g.integers(0, n, (2, 2000)))
    rp, col = csr.incoming_csr(ei, n)
    ref = numpy_csr(n, ei[1].numpy(), ei[0].numpy())
    np.testing.assert_array_equal(rp.numpy(), ref[0])
    np.testing.assert_array_equal(col.numpy(), ref[1])
    h, t = ei[0], ei[1]
    rp, col = csr.kg_csr(h, t, n, undirected=True)
    ref = numpy_csr(n, np.concatenate([h.numpy(), t.numpy()]),
                    np.concatenate([t.numpy(), h.numpy()]))
    np.testing.assert_array_equal(rp.numpy(), ref[0])
    np.testing.assert_array_equal(col.numpy(), ref[1])


def test_npz_round_trip(tmp_path):
    g = np.random.default_rng(5)
    rp, col = csr.build_csr(torch.from_numpy(g.integers(0, 100, 500)),
                            torch.from_numpy(g.integers(0, 100, 500)), 100)
    path = csr.save_csr(tmp_path / "graph", rp, col)
    assert path.name == "csr_adj.npz"
    with np.load(path) as z:
        assert set(z.files) == {"rowptr", "col"}
        assert z["rowptr"].dtype == np.int32 and z["col"].dtype == np.int32
    rp2, col2 = csr.load_csr(tmp_path / "graph")
    assert torch.equal(rp, rp2) and torch.equal(col, col2)


def test_bounds_are_checked(tmp_path):
    with pytest.raises(ValueError):
        csr.build_csr(torch.tensor([0, 5]), torch.tensor([1, 1]), 5)
    with pytest.raises(ValueError):
        csr.build_csr(torch.tensor([0, 1]), torch.tensor([1]), 5)
    bad = tmp_path / "bad.npz"
    np.savez(bad, rowptr=np.array([0, 3, 2], dtype=np.int32), col=np.zeros(2, np.int32))
    with pytest.raises(ValueError):
        csr.load_csr(bad)


@pytest.mark.gpu
def test_gpu_build_matches_cpu_build():
    g = torch.Generator().manual_seed(6)
    n, e = 2_000_000, 20_000_000
    rows = torch.randint(0, n, (e,), generator=g)
    nbrs = torch.randint(0, n, (e,), generator=g)
    rp_d, col_d = csr.build_csr(rows, nbrs, n, device="cuda")
    rp_c, col_c = csr.build_csr(rows, nbrs, n)
    assert torch.equal(rp_d.cpu(), rp_c) and torch.equal(col_d.cpu(), col_c)
