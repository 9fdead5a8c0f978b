"""Pure-PyTorch aggregation from sampled ids (the semantics of the
reference's tests/reference.py:19-45): mean over the valid (>= 0) ids of a
row, nested mean over non-empty first-hop slots, and the saved-index replay
gradients of tests/test_correctness.py:44-53 and tests/test_2hop.py:54-60.
Used as a second, independent check of the oracle on the CPU."""

from __future__ import annotations

import torch


def mean_from_samples(x: torch.Tensor, samples: torch.Tensor) -> torch.Tensor:
    out = x.new_zeros((samples.size(0), x.size(1)))
    for r in range(samples.size(0)):
        ids = samples[r][samples[r] >= 0].long()
        if ids.numel():
            out[r] = x[ids].mean(dim=0)
    return out


def nested_mean_from_samples(x: torch.Tensor, samples2: torch.Tensor) -> torch.Tensor:
    out = x.new_zeros((samples2.size(0), x.size(1)))
    for r in range(samples2.size(0)):
        means = []
        for i in range(samples2.size(1)):
            ids = samples2[r, i][samples2[r, i] >= 0].long()
            if ids.numel():
                means.append(x[ids].mean(dim=0))
        if means:
            out[r] = torch.stack(means).mean(dim=0)
    return out


def replay_grad_1hop(samples: torch.Tensor, grad_out: torch.Tensor, num_nodes: int) -> torch.Tensor:
    grad = grad_out.new_zeros((num_nodes, grad_out.size(1)))
    for r in range(samples.size(0)):
        ids = samples[r][samples[r] >= 0].long()
        if ids.numel():
            grad.index_add_(0, ids, (grad_out[r] / ids.numel()).expand(ids.numel(), -1))
    return grad


def replay_grad_2hop(samples2: torch.Tensor, grad_out: torch.Tensor, num_nodes: int) -> torch.Tensor:
    grad = grad_out.new_zeros((num_nodes, grad_out.size(1)))
    for r in range(samples2.size(0)):
        groups = [row[row >= 0].long() for row in samples2[r] if bool(row.ge(0).any())]
        for ids in groups:
            contrib = grad_out[r] / (len(groups) * ids.numel())
            grad.index_add_(0, ids, contrib.expand(ids.numel(), -1))
    return grad


def assert_unique_valid(samples: torch.Tensor) -> None:
    if samples.numel() == 0:
        return
    for row in samples.reshape(-1, samples.size(-1)):
        ids = row[row >= 0]
        assert ids.unique().numel() == ids.numel()
