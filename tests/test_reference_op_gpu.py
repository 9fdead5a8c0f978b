"""Differential test against the reference's own CUDA op on the same B200.

The reference op (fuseop, built from the reference sources into
oracle/_ref/fuseop by ``python -m oracle.build --ref``) and this package run
on identical device inputs; sampled ids and forward outputs must be
bit-identical, feature gradients equal within rtol 1e-5 / atol 1e-6.
Includes the full-size 2-hop benchmark graph (N=2.45M, ~123M edges).
"""

from __future__ import annotations

import functools
import importlib.util
import sys
from pathlib import Path

import pytest
import torch

import fusesampleagg_b200 as fsa
from fusesampleagg_b200 import synthetic
from tests.golden import cases as C

pytestmark = pytest.mark.gpu

REF_DIR = Path(__file__).resolve().parents[1] / "oracle" / "_ref"
RTOL, ATOL = 1e-5, 1e-6


@functools.lru_cache(maxsize=None)
def ref():
    if not (REF_DIR / "fuseop" / "__init__.py").exists():
        pytest.skip("reference op not built (python -m oracle.build --ref)")
    spec = importlib.util.spec_from_file_location(
        "fuseop", REF_DIR / "fuseop" / "__init__.py",
        submodule_search_locations=[str(REF_DIR / "fuseop")])
    mod = importlib.util.module_from_spec(spec)
    # Registered under its own name only while it imports its _C extension;
    # afterwards `fuseop` in this process is this repository's package again.
    prev = sys.modules.get("fuseop")
    sys.modules["fuseop"] = mod
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.modules.pop("fuseop._C", None)
        if prev is not None:
            sys.modules["fuseop"] = prev
        else:
            del sys.modules["fuseop"]
    return mod


@functools.lru_cache(maxsize=None)
def graph(name):
    if name == "c2":
        w = synthetic.WORKLOADS["c2_2hop_powerlaw"]
        g = w.graph(0, "cuda")
        return g.rowptr, g.col, g.num_nodes
    g = C.GRAPHS[name]()
    return g.rowptr.cuda(), g.col.cuda(), g.num_nodes


def roots(name, n, batch, seed):
    if name == "c2":
        return synthetic.root_batch(n, batch, seed, device="cuda")
    return C.frontier_for(name, C.GRAPHS[name](), batch, seed).cuda()


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.int32), b.contiguous().view(torch.int32))


@pytest.mark.parametrize("name", ["toy", "hub", "uniform", "powerlaw", "c2"])
@pytest.mark.parametrize("fan,seed", [((15, 10), 0), ((15, 10), 1), ((25, 10), 3), ((8, 4), 9)])
def test_2hop_matches_reference_op(name, fan, seed):
    rp, cl, n = graph(name)
    x = synthetic.features(n, 100, seed=1, device="cuda")
    fr = roots(name, n, 1024 if name == "c2" else 128, seed)
    mine = fsa.fused_sample_agg_2hop_with_samples(rp, cl, x, fr, *fan, replay_seed=seed)
    theirs = ref().fused_sample_agg_2hop_with_samples(rp, cl, x, fr, *fan, replay_seed=seed)
    assert torch.equal(mine[1], theirs[1])
    assert torch.equal(mine[2], theirs[2])
    assert same_bits(mine[0], theirs[0])


@pytest.mark.parametrize("name", ["toy", "hub", "uniform", "powerlaw", "c2"])
@pytest.mark.parametrize("k,seed", [(10, 0), (8, 1234), (1024, 5)])
def test_1hop_matches_reference_op(name, k, seed):
    rp, cl, n = graph(name)
    x = synthetic.features(n, 128, seed=1, device="cuda")
    fr = roots(name, n, 1024 if name == "c2" else 128, seed)
    mine = fsa.fused_sample_agg_with_samples(rp, cl, x, fr, k, replay_seed=seed)
    theirs = ref().fused_sample_agg_with_samples(rp, cl, x, fr, k, replay_seed=seed)
    assert torch.equal(mine[1], theirs[1])
    assert torch.equal(mine[2], theirs[2])
    assert same_bits(mine[0], theirs[0])


@pytest.mark.parametrize("name,hops", [("powerlaw", 1), ("powerlaw", 2), ("c2", 2), ("hub", 2)])
def test_gradients_match_reference_op(name, hops):
    rp, cl, n = graph(name)
    x = synthetic.features(n, 100, seed=1, device="cuda")
    fr = roots(name, n, 1024 if name == "c2" else 128, 4)
    go = synthetic.features(fr.numel(), 100, seed=2, device="cuda")
    grads = []
    for mod in (fsa, ref()):
        xg = x.clone().requires_grad_(True)
        if hops == 1:
            y = mod.fused_sample_agg(rp, cl, xg, fr, 10, replay_seed=11)
        else:
            y = mod.fused_sample_agg_2hop(rp, cl, xg, fr, 15, 10, replay_seed=11)
        y.backward(go)
        grads.append(xg.grad)
    torch.testing.assert_close(grads[0], grads[1], rtol=RTOL, atol=ATOL)
