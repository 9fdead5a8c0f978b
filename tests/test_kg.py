"""Knowledge-graph encoder step (fusesampleagg_b200/kg.py).

CPU: the model wiring with a stand-in aggregation (shapes, unique/inverse
bookkeeping, gradients reaching every parameter).  GPU: the training step on
the C4a shapes with this package's operator and with the reference op from
the same initial state — first loss bit-identical (the operator's outputs
are), later losses within fp32 atomic-order tolerance."""

from __future__ import annotations

import pytest
import torch

from fusesampleagg_b200 import kg


def standin_op(rowptr, col, x, frontier, f1, f2, replay_seed=0):
    # test-only stand-in: mean of the first neighbour's row (no sampling)
    first = col[rowptr[frontier.long()].clamp(max=col.numel() - 1)].long()
    return x[first]


def test_encoder_wiring_on_cpu():
    torch.manual_seed(0)
    n, d = 50, 8
    rowptr = torch.arange(0, 2 * (n + 1), 2, dtype=torch.int32)
    col = torch.randint(0, n, (2 * n,), dtype=torch.int32)
    m = kg.KGEncoder(n, 4, d)
    ids = torch.tensor([3, 7, 3, 9, 7])
    z = m.encode(ids, rowptr, col, 2, 2, 0, standin_op)
    assert z.shape == (5, d)
    assert torch.equal(z[0], z[2]) and torch.equal(z[1], z[4])
    loss = m.score(z, m.relations(torch.zeros(5, dtype=torch.long)), z).sum()
    loss.backward()
    assert all(p.grad is not None for p in m.parameters())


@pytest.mark.gpu
def test_kg_step_matches_reference_op():
    from tests.test_reference_op_gpu import ref

    r = ref()
    losses = {}
    for name, op in (("ours", kg.load_op("ours")), ("reference", r.fused_sample_agg_2hop)):
        torch.manual_seed(0)
        data = kg.KGData("c4a_kg_2hop", seed=0)
        model = kg.KGEncoder(data.num_entities, data.num_relations, data.workload.dim).cuda()
        step, _ = kg.make_train_step(model, data, op, data.workload.fanouts, 512, 16)
        losses[name] = [step(i) for i in range(3)]
    a, b = losses["ours"], losses["reference"]
    assert torch.equal(a[0], b[0])
    torch.testing.assert_close(torch.stack(a), torch.stack(b), rtol=1e-4, atol=1e-5)
