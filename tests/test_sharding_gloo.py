"""Multi-rank root partitioning on CPU (gloo, world size 2 and 3).

Each rank samples its slice of the global batch with batch_offset = slice
start (through the oracle, which follows the same seed rule as the device
kernels); the gathered ids must equal a single-process run of the whole
batch, and the all-reduced per-rank gradients must equal the whole-batch
gradient.  Also covers a rank that fails: the others see the error instead
of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fusesampleagg_b200 import sharding


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_covers_batch_exactly():
    for batch in (0, 1, 7, 1024, 1025):
        for world in (1, 2, 3, 8):
            spans = [sharding.partition(batch, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.partition(4, 2, 2)


def _graph():
    from tests.golden import cases as C

    return C.powerlaw_graph()


def _worker(rank, world, port, out_dir, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        from fusesampleagg_b200 import synthetic
        from oracle import oracle

        g = _graph()
        frontier = synthetic.root_batch(g.num_nodes, 101, seed=3)
        mine, off = sharding.local_roots(frontier, rank, world)
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        s1, s2 = oracle.sample_2hop(g.rowptr.numpy(), g.col.numpy(), mine.numpy(), 15, 10, 77,
                                    batch_offset=off)
        go = synthetic.features(frontier.numel(), 6, seed=2)[off:off + mine.numel()]
        grad = torch.from_numpy(oracle.backward_2hop(go.numpy(), s1, s2, g.num_nodes))
        gathered = [None] * world
        dist.all_gather_object(gathered, (off, s1, s2))
        sharding.allreduce_gradient(grad)
        if rank == 0:
            np.save(os.path.join(out_dir, "grad.npy"), grad.numpy())
            parts = sorted(gathered, key=lambda t: t[0])
            np.save(os.path.join(out_dir, "s1.npy"), np.concatenate([p[1] for p in parts]))
            np.save(os.path.join(out_dir, "s2.npy"), np.concatenate([p[2] for p in parts]))
    finally:
        if rank == fail_rank:
            os._exit(3)
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ranks_reproduce_single_process_batch(world, tmp_path):
    from fusesampleagg_b200 import synthetic
    from oracle import oracle

    mp.start_processes(_worker, args=(world, free_port(), str(tmp_path), -1), nprocs=world,
                       start_method="spawn")
    g = _graph()
    frontier = synthetic.root_batch(g.num_nodes, 101, seed=3)
    s1, s2 = oracle.sample_2hop(g.rowptr.numpy(), g.col.numpy(), frontier.numpy(), 15, 10, 77)
    np.testing.assert_array_equal(np.load(tmp_path / "s1.npy"), s1)
    np.testing.assert_array_equal(np.load(tmp_path / "s2.npy"), s2)
    go = synthetic.features(frontier.numel(), 6, seed=2)
    whole = oracle.backward_2hop(go.numpy(), s1, s2, g.num_nodes)
    np.testing.assert_allclose(np.load(tmp_path / "grad.npy"), whole, rtol=1e-5, atol=1e-6)


def test_failed_rank_surfaces_as_error(tmp_path):
    with pytest.raises(Exception):
        mp.start_processes(_worker, args=(2, free_port(), str(tmp_path), 1), nprocs=2,
                           start_method="spawn")


def test_exchange_bytes_helper():
    """Region size of the owner-computed backward / gradient exchange: the C
    ABI's layout; invalid sizes raise before anything is allocated."""
    from fusesampleagg_b200 import sharding

    assert sharding.exchange_bytes(1024, 15, 10, 100) == 256 + 1024 * (672 + 400)
    assert sharding.exchange_bytes(0, 15, 10, 100) == 256
    with pytest.raises(ValueError):
        sharding.exchange_bytes(-1, 15, 10, 100)
    with pytest.raises(ValueError):
        sharding.exchange_bytes(8, 5, 2400, 16)  # over the 12000-entry limit
