"""Row-sharded features over two GPUs (one process per GPU, NCCL, CUDA IPC
peer mappings): the sharded 2-hop op must give the ids and outputs of the
unsharded op on the whole table bit for bit, and its gradient shards must
equal the rows of the all-reduced unsharded gradient (rtol 1e-5 / atol
1e-6), with the backward sent as remote red.adds (push), computed by the
owners from the exchange regions (pull), and with the shard kept across
steps and only its touched rows cleared (persistent).  Skipped with fewer than two GPUs;
host-side pieces are also covered on the CPU."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch

from fusesampleagg_b200 import sharding

RTOL, ATOL = 1e-5, 1e-6


def test_shard_spans_partition_rows():
    for n in (1, 5, 10, 1000, 1001):
        for world in (1, 2, 3, 8):
            spans = [sharding.shard_span(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            rows = -(-n // world)
            assert all(b - a <= rows for a, b in spans)
    with pytest.raises(ValueError):
        sharding.shard_span(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, dim, fans, mode, results):
    import numpy as np  # noqa: F401
    import torch.distributed as dist

    import fusesampleagg_b200 as fsa
    from fusesampleagg_b200 import synthetic
    from tests.golden import cases as C

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    feats = None
    try:
        g = C.powerlaw_graph()
        rp, cl = g.rowptr.to(dev), g.col.to(dev)
        n = g.num_nodes
        x = synthetic.features(n, dim, seed=1, device=dev)
        start, stop = sharding.shard_span(n, rank, world)
        local = x[start:stop].clone().requires_grad_(True)
        roots = synthetic.root_batch(n, 256, seed=3, device=dev)
        mine, off = sharding.local_roots(roots, rank, world)
        k1, k2 = fans
        ex = sharding.exchange_bytes(-(-256 // world), k1, k2, dim) if mode != "push" else 0
        feats = sharding.ShardedFeatures(local, n, exchange_bytes=ex,
                                         persistent=mode == "persistent")
        go = synthetic.features(mine.numel(), dim, seed=5 + rank, device=dev)
        ok = True
        for step in range(3):  # the shard is re-zeroed (or its touched rows cleared) each step
            out = sharding.fused_sample_agg_2hop_sharded(rp, cl, feats, mine, k1, k2,
                                                         replay_seed=17 + step,
                                                         batch_offset=off)
            out.backward(go)
            xr = x.clone().requires_grad_(True)
            ref = fsa.fused_sample_agg_2hop(rp, cl, xr, mine, k1, k2, replay_seed=17 + step,
                                            batch_offset=off)
            ref.backward(go)
            full = xr.grad.clone()
            dist.all_reduce(full)
            torch.cuda.synchronize()
            ok &= torch.equal(out.view(torch.int32), ref.detach().view(torch.int32))
            ok &= torch.allclose(feats.grad, full[start:stop], rtol=RTOL, atol=ATOL)
        with torch.no_grad():
            o2, s1, s2 = sharding._forward_2hop_sharded(rp, cl, feats, mine, k1, k2, 99, True,
                                                        off, None)
            r2, t1, t2 = fsa.fused_sample_agg_2hop_with_samples(rp, cl, x, mine, k1, k2, 99,
                                                                batch_offset=off)
        ok &= torch.equal(s1, t1) and torch.equal(s2, t2)
        ok &= torch.equal(o2.view(torch.int32), r2.view(torch.int32))
        results[rank] = bool(ok)
    finally:
        if feats is not None:
            feats.close()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["push", "pull", "persistent"])
@pytest.mark.parametrize("dim,fans", [(64, (15, 10)), (33, (8, 4))])
def test_sharded_two_gpus_match_unsharded(dim, fans, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_worker, args=(world, _free_port(), dim, fans, mode, results), nprocs=world,
                 join=True)
        assert dict(results) == {0: True, 1: True}


def _exchange_worker(rank, world, port, persistent, results):
    import torch.distributed as dist

    import fusesampleagg_b200 as fsa
    from fusesampleagg_b200 import synthetic
    from tests.golden import cases as C

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    ex = None
    try:
        g = C.powerlaw_graph()
        rp, cl = g.rowptr.to(dev), g.col.to(dev)
        n, dim, (k1, k2) = g.num_nodes, 48, (15, 10)
        x = synthetic.features(n, dim, seed=1, device=dev)
        roots = synthetic.root_batch(n, 256, seed=4, device=dev)
        mine, off = sharding.local_roots(roots, rank, world)
        ex = sharding.GradientExchange(n, dim, sharding.exchange_bytes(-(-256 // world), k1, k2,
                                                                        dim), device=dev,
                                       persistent=persistent)
        ok = True
        for step in range(3):
            go = synthetic.features(mine.numel(), dim, seed=20 + 2 * rank + step, device=dev)
            xe = x.clone().requires_grad_(True)
            out = sharding.fused_sample_agg_2hop_exchange(rp, cl, xe, mine, k1, k2,
                                                          replay_seed=step, batch_offset=off,
                                                          exchange=ex)
            out.backward(go)
            xr = x.clone().requires_grad_(True)
            ref = fsa.fused_sample_agg_2hop(rp, cl, xr, mine, k1, k2, replay_seed=step,
                                            batch_offset=off)
            ref.backward(go)
            full = xr.grad.clone()
            dist.all_reduce(full)
            torch.cuda.synchronize()
            ok &= torch.equal(out.view(torch.int32), ref.detach().view(torch.int32))
            got = ex.grad if persistent else xe.grad
            ok &= (xe.grad is None) == persistent
            ok &= torch.allclose(got, full, rtol=RTOL, atol=ATOL)
        results[rank] = bool(ok)
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("persistent", [False, True], ids=["fresh", "persistent"])
def test_gradient_exchange_two_gpus_equals_allreduce(persistent):
    """Replicated features: the exchange backward leaves every rank with the
    all-reduced gradient of the per-rank gradients."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_exchange_worker, args=(world, _free_port(), persistent, results), nprocs=world,
                 join=True)
        assert dict(results) == {0: True, 1: True}

