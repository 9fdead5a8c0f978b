"""The forward-only microbenchmark (fusesampleagg_b200/microbench_2hop.py):
its workload generator on the CPU, and on the GPU the sampled ids on that
workload against the oracle plus the JSON fields of a short run."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fusesampleagg_b200 import microbench_2hop as mb


def test_regular_graph_layout():
    torch.manual_seed(0)
    rowptr, col = mb.regular_graph(1000, 20, device="cpu")
    assert rowptr.dtype == torch.int32 and col.dtype == torch.int32
    assert rowptr.numel() == 1001 and int(rowptr[-1]) == col.numel() == 20_000
    assert bool((rowptr[1:] - rowptr[:-1] == 20).all())
    assert int(col.min()) >= 0 and int(col.max()) < 1000


def test_inputs_are_seeded():
    a = mb.make_inputs(500, 8, 5, 64, seed=3, device="cpu")
    b = mb.make_inputs(500, 8, 5, 64, seed=3, device="cpu")
    for u, v in zip(a, b):
        assert torch.equal(u, v)


@pytest.mark.gpu
def test_microbench_workload_ids_match_oracle():
    import fusesampleagg_b200 as fsa
    from oracle import oracle

    rowptr, col, x, roots = mb.make_inputs(20_000, 32, 20, 512, seed=1234)
    out, s1, s2 = fsa.fused_sample_agg_2hop_with_samples(rowptr, col, x, roots, 15, 10, 1254)
    r1, r2 = oracle.sample_2hop(rowptr.cpu().numpy(), col.cpu().numpy(), roots.cpu().numpy(),
                                15, 10, 1254)
    np.testing.assert_array_equal(s1.cpu().numpy(), r1)
    np.testing.assert_array_equal(s2.cpu().numpy(), r2)
    ref_out = oracle.forward_2hop(x.cpu().numpy(), r2)
    assert np.array_equal(out.cpu().numpy().view(np.int32), ref_out.view(np.int32))


@pytest.mark.gpu
def test_microbench_run_fields():
    res = mb.run(type("A", (), dict(nodes=10_000, features=16, degree=20, batch_size=256,
                                    fanout=[15, 10], steps=3, warmup=3, seed=1234,
                                    impl="ours"))())
    assert res["steps"] == 3 and res["mean_step_ms"] > 0
    assert res["sampled_edges_per_second"] == pytest.approx(
        256 * 150 * 3 / (res["mean_step_ms"] * 3 / 1000.0))


@pytest.mark.gpu
def test_microbench_kernel_times():
    res = mb.run(type("A", (), dict(nodes=10_000, features=16, degree=20, batch_size=256,
                                    fanout=[15, 10], steps=3, warmup=3, seed=1234,
                                    impl="ours", kernel_times=True))())
    k = res["kernels"]
    # degree 20 >= both fanouts: every slot holds a valid leaf
    assert k["valid_leaves"] == 256 * 150
    assert k["gather_algorithmic_bytes"] == 4 * 256 * 150 * (1 + 1 + 16) + 4 * 16 * 256
    for name in ("plan_us", "draw_us", "gather_us"):
        assert k[name] > 0
    assert k["gather_gbs"] > 0 and k["peak_gbs"] > 0
