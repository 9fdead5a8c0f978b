"""fsa_sample_agg_2hop_forward_noalloc (library-owned static scratch) against
the workspace entry point fsa_sample_agg_2hop_forward, both through the C ABI.

The two entry points run the same kernels, so outputs and sampled ids must be
bit-identical (the forward tolerance of every 2-hop parity test).  The calls
come in a row with different shapes, so stale scratch from the previous call
would show.  The file sorts last so that it also runs after every other test
has used the library.
"""

from __future__ import annotations

import functools

import pytest
import torch

from fusesampleagg_b200 import _lib, synthetic
from tests.golden import cases as C

L = _lib.LIB
U64_MAX = (1 << 64) - 1


def ptr(t):
    return None if t is None else t.data_ptr()


@functools.lru_cache(maxsize=None)
def dev_case(graph_name, batch, root_seed, dim):
    g = C.GRAPHS[graph_name]()
    fr = C.frontier_for(graph_name, g, batch, root_seed)
    x = synthetic.features(g.num_nodes, dim, seed=1)
    return g, g.rowptr.cuda(), g.col.cuda(), x.cuda(), fr.cuda()


def forward(noalloc, graph_name, batch, root_seed, dim, k1, k2, seed, want_ids, zero=None):
    g, rp, cl, x, fr = dev_case(graph_name, batch, root_seed, dim)
    B = fr.numel()
    out = torch.full((B, dim), float("nan"), device="cuda")
    s1 = torch.full((B, k1), -7, dtype=torch.int32, device="cuda") if want_ids else None
    s2 = torch.full((B, k1, k2), -7, dtype=torch.int32, device="cuda") if want_ids else None
    stream = torch.cuda.current_stream().cuda_stream
    zc = 0 if zero is None else zero.numel()
    head = (ptr(rp), ptr(cl), g.num_nodes, g.num_edges, ptr(x), dim, ptr(fr), B, 0, k1, k2, seed,
            ptr(out), ptr(s1), ptr(s2))
    if noalloc:
        st = L.fsa_sample_agg_2hop_forward_noalloc(*head, ptr(zero), zc, stream)
    else:
        nbytes = L.fsa_sample_agg_2hop_workspace_size(B, k1, k2, int(want_ids), int(want_ids))
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
        st = L.fsa_sample_agg_2hop_forward(*head, ptr(ws), nbytes, ptr(zero), zc, stream)
    _lib.check(st, "2-hop forward")
    torch.cuda.synchronize()
    return out, s1, s2


def assert_same(a, b):
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))


# (graph, batch, root seed, dim, fanout1, fanout2, seed, ids requested)
CALL_A = ("powerlaw", 256, 0, 100, 15, 10, 0, False)
CALL_B = ("hub", 48, 4, 33, 25, 10, U64_MAX, True)
CALL_MAX = ("powerlaw", 3500, 5, 16, 15, 10, 77, False)


@pytest.mark.gpu
def test_two_calls_in_a_row_match_workspace_entry_point():
    for call in (CALL_A, CALL_B):
        got = forward(True, *call)
        want = forward(False, call[0], *call[1:7], True)
        assert_same(got[0], want[0])
        if call[7]:
            assert torch.equal(got[1], want[1]) and torch.equal(got[2], want[2])


@pytest.mark.gpu
def test_repeat_call_is_identical_and_fills_zero_buffer():
    g, *_ = dev_case("powerlaw", 256, 0, 100)
    zero = torch.ones(g.num_nodes * 100, device="cuda")
    first = forward(True, *CALL_A[:7], True, zero=zero)
    assert int(torch.count_nonzero(zero)) == 0
    second = forward(True, *CALL_A[:7], True)
    assert_same(first[0], second[0])
    assert torch.equal(first[1], second[1]) and torch.equal(first[2], second[2])
    assert bool((first[1] >= -1).all()) and bool((first[2] >= -1).all())


@pytest.mark.gpu
def test_largest_batch_within_scratch():
    _, b, _, _, k1, k2, _, ids = CALL_MAX
    need = L.fsa_sample_agg_2hop_workspace_size(b, k1, k2, int(ids), int(ids))
    assert 0.75 * _lib.NOALLOC_SCRATCH_BYTES < need <= _lib.NOALLOC_SCRATCH_BYTES
    got = forward(True, *CALL_MAX)
    want = forward(False, *CALL_MAX[:7], True)
    assert_same(got[0], want[0])


# Stand-in device addresses for the host-side checks below: non-null and
# aligned, never dereferenced (every call returns before any CUDA call).
FAKE = 1 << 20


def test_oversized_call_is_rejected_before_cuda():
    """Runs without a GPU: the size check precedes every CUDA call."""
    b = 10_000
    assert L.fsa_sample_agg_2hop_workspace_size(b, 15, 10, 1, 1) > _lib.NOALLOC_SCRATCH_BYTES
    st = L.fsa_sample_agg_2hop_forward_noalloc(FAKE, FAKE, 10, 10, FAKE, 4, FAKE, b, 0, 15, 10,
                                               1, FAKE, None, None, None, 0, None)
    assert st == _lib.FSA_ERR_SCRATCH_LIMIT
    assert b"scratch" in L.fsa_status_string(st)
    # batch sizes far beyond the scratch never reach the layout arithmetic
    st = L.fsa_sample_agg_2hop_forward_noalloc(FAKE, FAKE, 10, 10, FAKE, 4, FAKE, 1 << 62, 0,
                                               1, 1, 1, FAKE, None, None, None, 0, None)
    assert st == _lib.FSA_ERR_SCRATCH_LIMIT
    # no sampling work: no scratch, same result as the workspace entry point
    assert L.fsa_sample_agg_2hop_forward_noalloc(None, None, 10, 10, None, 4, None, 5, 0, 0, 3,
                                                 1, None, None, None, None, 0,
                                                 None) == _lib.FSA_OK


@pytest.mark.parametrize("bad", [
    {"rowptr": None},                   # null graph pointer
    {"out": None},                      # null output
    {"offset": -1},                     # negative batch_offset
    {"zero_count": 8},                  # zero_count > 0 with no zero_fill
    {"k2": 12000},                      # fanout pair over the entry limit
])
def test_oversized_call_with_bad_arguments_is_invalid_argument(bad):
    """Runs without a GPU: arguments are checked before the size limit, so a
    call that is both too large and malformed is told it is malformed."""
    a = {"rowptr": FAKE, "out": FAKE, "offset": 0, "zero_count": 0, "k2": 10}
    a.update(bad)
    st = L.fsa_sample_agg_2hop_forward_noalloc(a["rowptr"], FAKE, 10, 10, FAKE, 4, FAKE, 10_000,
                                               a["offset"], 15, a["k2"], 1, a["out"], None, None,
                                               None, a["zero_count"], None)
    assert st == _lib.FSA_ERR_INVALID_ARGUMENT
