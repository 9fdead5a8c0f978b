"""Pins the CPU oracle to the reference's own CUDA op.

tests/golden/reference_b200.{npz,json} were recorded by
tests/golden/make_golden.py from the reference op (its own sources built for
sm_100) on a B200.  The oracle must reproduce every sampled id and take
count bit for bit, every forward output bit for bit (SHA-256 of the fp32
bytes), and the recorded gradients within rtol 1e-5 / atol 1e-6 (the
reference accumulates with atomics in a nondeterministic order).
"""

from __future__ import annotations

import functools
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle
from tests.golden import cases as C

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "reference_b200.json").read_text())
ARRAYS = np.load(GOLDEN / "reference_b200.npz")
CASES = {c["name"]: c for c in C.CASES}


@functools.lru_cache(maxsize=None)
def graph(name):
    return C.GRAPHS[name]()


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_fixture_covers_every_case():
    assert set(META["cases"]) == set(CASES)
    assert "B200" in META["gpu"]


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_reproduces_reference_op(name):
    case = CASES[name]
    rec = META["cases"][name]
    g = graph(case["graph"])
    assert g.digest() == rec["graph_digest"], "graph generator drifted from the fixture"
    fr = C.frontier_for(case["graph"], g, case["batch"], case["root_seed"])
    assert sha(fr.numpy()) == rec["frontier_sha"]
    x = C.features_for(case, g.num_nodes).numpy()
    rp, cl, frn = g.rowptr.numpy(), g.col.numpy(), fr.numpy()
    if case["hops"] == 1:
        (k,) = case["fanouts"]
        s, t = oracle.sample_1hop(rp, cl, frn, k, case["seed"])
        np.testing.assert_array_equal(s, ARRAYS[f"{name}/samples"])
        np.testing.assert_array_equal(t, ARRAYS[f"{name}/takes"])
        out = oracle.forward_1hop(x, s, t)
    else:
        k1, k2 = case["fanouts"]
        s1, s2 = oracle.sample_2hop(rp, cl, frn, k1, k2, case["seed"])
        np.testing.assert_array_equal(s1, ARRAYS[f"{name}/samples1"])
        np.testing.assert_array_equal(s2, ARRAYS[f"{name}/samples2"])
        out = oracle.forward_2hop(x, s2)
    if case["store_out"]:
        np.testing.assert_array_equal(out.view(np.int32), ARRAYS[f"{name}/out"].view(np.int32))
    assert sha(out) == rec["out_sha"], "forward output is not bit-identical to the reference op"
    if case["grad"]:
        go = C.grad_out_for(case, frn.size).numpy()
        if case["hops"] == 1:
            grad = oracle.backward_1hop(s, t, go, g.num_nodes)
        else:
            grad = oracle.backward_2hop(go, s1, s2, g.num_nodes)
        np.testing.assert_allclose(grad, ARRAYS[f"{name}/grad_x"], rtol=1e-5, atol=1e-6)
