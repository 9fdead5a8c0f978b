"""The CPU oracle against the reference's documented semantics: means from
the saved ids (pure PyTorch), without-replacement reservoirs, -1 padding,
take counts, the 2-hop zero-fanout convention, replay gradients, the
batch-offset rule, and the statistics of Algorithm R."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fusesampleagg_b200 import synthetic
from oracle import oracle
from tests import torch_reference as R
from tests.golden import cases as C


@pytest.fixture(scope="module")
def toy():
    return C.toy_graph()


@pytest.fixture(scope="module")
def pl():
    return C.powerlaw_graph()


def arrays(g):
    return g.rowptr.numpy(), g.col.numpy()


@pytest.mark.parametrize("k", [0, 1, 2, 5, 6, 9])
@pytest.mark.parametrize("dim", [1, 8, 31, 32, 33, 129])
def test_1hop_forward_is_mean_of_saved_samples(toy, k, dim):
    rp, cl = arrays(toy)
    fr = C.frontier_for("toy", toy, 0, 0).numpy()
    x = synthetic.features(toy.num_nodes, dim, seed=1)
    s, t = oracle.sample_1hop(rp, cl, fr, k, 17)
    out = oracle.forward_1hop(x.numpy(), s, t)
    torch.testing.assert_close(torch.from_numpy(out), R.mean_from_samples(x, torch.from_numpy(s)))
    np.testing.assert_array_equal(t, (s >= 0).sum(axis=1))
    R.assert_unique_valid(torch.from_numpy(s))


def test_rows_shorter_than_fanout_keep_row_order_and_pad(toy):
    rp, cl = arrays(toy)
    fr = np.arange(8, dtype=np.int32)
    s, t = oracle.sample_1hop(rp, cl, fr, 7, 3)
    for r in range(8):
        row = cl[rp[r]:rp[r + 1]]
        assert t[r] == len(row)
        np.testing.assert_array_equal(s[r, :len(row)], row)
        assert (s[r, len(row):] == -1).all()


def test_samples_are_row_members_and_unique(pl):
    rp, cl = arrays(pl)
    fr = synthetic.root_batch(pl.num_nodes, 300, seed=9).numpy()
    s, t = oracle.sample_1hop(rp, cl, fr, 25, 4)
    for b, r in enumerate(fr):
        row = set(cl[rp[r]:rp[r + 1]].tolist())
        ids = s[b, :t[b]]
        assert set(ids.tolist()) <= row
        assert len(set(ids.tolist())) == t[b] == min(len(row), 25)


@pytest.mark.parametrize("fan", [(3, 2), (15, 10), (2, 7)])
@pytest.mark.parametrize("dim", [1, 16, 127, 129])
def test_2hop_forward_is_nested_mean(pl, fan, dim):
    rp, cl = arrays(pl)
    fr = synthetic.root_batch(pl.num_nodes, 40, seed=1).numpy()
    x = synthetic.features(pl.num_nodes, dim, seed=1)
    s1, s2 = oracle.sample_2hop(rp, cl, fr, *fan, 1234)
    out = oracle.forward_2hop(x.numpy(), s2)
    torch.testing.assert_close(torch.from_numpy(out),
                               R.nested_mean_from_samples(x, torch.from_numpy(s2)))
    R.assert_unique_valid(torch.from_numpy(s1))
    R.assert_unique_valid(torch.from_numpy(s2))


def test_2hop_second_hop_rows_follow_first_hop(pl):
    rp, cl = arrays(pl)
    fr = synthetic.root_batch(pl.num_nodes, 50, seed=2).numpy()
    s1, s2 = oracle.sample_2hop(rp, cl, fr, 15, 10, 8)
    for b in range(fr.size):
        for i in range(15):
            m = s1[b, i]
            if m < 0:
                assert (s2[b, i] == -1).all()
            else:
                row = set(cl[rp[m]:rp[m + 1]].tolist())
                ids = s2[b, i][s2[b, i] >= 0]
                assert set(ids.tolist()) <= row and ids.size == min(len(row), 10)


@pytest.mark.parametrize("fan", [(0, 0), (0, 2), (2, 0)])
def test_2hop_zero_fanouts_give_zero_and_minus_one(toy, fan):
    rp, cl = arrays(toy)
    fr = C.frontier_for("toy", toy, 0, 0).numpy()
    s1, s2 = oracle.sample_2hop(rp, cl, fr, *fan, 1)
    assert (s1 == -1).all() and (s2 == -1).all()
    out = oracle.forward_2hop(np.ones((8, 4), np.float32), s2)
    assert not out.any()


def test_second_hop_seed_ignores_batch_index(pl):
    """Second-hop streams depend on (seed, root, slot) only, so a root's
    second-hop rows for a given first-hop result do not move with its batch
    position (fused_sample_agg.cu:170-171); first-hop rows do."""
    rp, cl = arrays(pl)
    root = np.array([int(np.argmax(np.diff(rp)))], dtype=np.int32)
    a1, a2 = oracle.sample_2hop(rp, cl, root, 15, 10, 5, batch_offset=0)
    b1, b2 = oracle.sample_2hop(rp, cl, root, 15, 10, 5, batch_offset=1)
    assert not np.array_equal(a1, b1)
    for i in range(15):
        for j in range(15):
            if a1[0, i] == b1[0, j] and i == j:
                np.testing.assert_array_equal(a2[0, i], b2[0, j])


def test_batch_offset_equals_slicing(pl):
    rp, cl = arrays(pl)
    fr = synthetic.root_batch(pl.num_nodes, 64, seed=3).numpy()
    s_all, t_all = oracle.sample_1hop(rp, cl, fr, 10, 6)
    s_part, t_part = oracle.sample_1hop(rp, cl, fr[20:], 10, 6, batch_offset=20)
    np.testing.assert_array_equal(s_all[20:], s_part)
    a1, a2 = oracle.sample_2hop(rp, cl, fr, 15, 10, 6)
    p1, p2 = oracle.sample_2hop(rp, cl, fr[33:], 15, 10, 6, batch_offset=33)
    np.testing.assert_array_equal(a1[33:], p1)
    np.testing.assert_array_equal(a2[33:], p2)


def test_threads_do_not_change_results(pl):
    rp, cl = arrays(pl)
    fr = synthetic.root_batch(pl.num_nodes, 128, seed=4).numpy()
    a = oracle.sample_2hop(rp, cl, fr, 15, 10, 2, threads=1)
    b = oracle.sample_2hop(rp, cl, fr, 15, 10, 2, threads=4)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def test_replay_gradients_match_index_add(pl):
    rp, cl = arrays(pl)
    fr = synthetic.root_batch(pl.num_nodes, 60, seed=5).numpy()
    go = synthetic.features(60, 7, seed=2)
    s, t = oracle.sample_1hop(rp, cl, fr, 10, 42)
    g1 = oracle.backward_1hop(s, t, go.numpy(), pl.num_nodes)
    torch.testing.assert_close(torch.from_numpy(g1),
                               R.replay_grad_1hop(torch.from_numpy(s), go, pl.num_nodes))
    s1, s2 = oracle.sample_2hop(rp, cl, fr, 15, 10, 42)
    g2 = oracle.backward_2hop(go.numpy(), s1, s2, pl.num_nodes)
    torch.testing.assert_close(torch.from_numpy(g2),
                               R.replay_grad_2hop(torch.from_numpy(s2), go, pl.num_nodes))


def test_algorithm_r_inclusion_is_uniform():
    """Each of 20 neighbours is kept with probability 5/20 (chi-square over
    4000 rows, each its own seed stream via the batch index)."""
    deg, k, rows = 20, 5, 4000
    rowptr = np.array([0, deg], dtype=np.int32)
    col = np.arange(deg, dtype=np.int32)
    fr = np.zeros(rows, dtype=np.int32)
    s, _ = oracle.sample_1hop(rowptr, col, fr, k, 2024)
    counts = np.bincount(s.ravel(), minlength=deg)
    expected = rows * k / deg
    chi2 = float(((counts - expected) ** 2 / expected).sum())
    assert chi2 < 45.0  # 19 dof, p ~ 1e-3
