"""Root partitioning across GPUs (one process per GPU).

Roots are independent units: every root's samples depend only on the graph,
the replay seed, the root id and its index in the global batch (first-hop
seeds, fuseop/fused_sample_agg.cu:82-83 and :155-156; second-hop seeds use
the first-hop slot only, :170-171).  A rank that processes the contiguous
slice [start, stop) of the global batch with ``batch_offset=start`` therefore
draws exactly the ids a single GPU would draw for the whole batch, and the
forward needs no communication.

The feature gradient of a global batch is the sum of the ranks' gradients;
``allreduce_gradient`` is the optional NCCL all-reduce that turns per-rank
gradients into the global one for replicated embeddings.
"""

from __future__ import annotations

import torch


def partition(batch_size: int, rank: int, world: int) -> tuple[int, int]:
    """Balanced contiguous slice [start, stop) of a global batch for `rank`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if batch_size < 0:
        raise ValueError("batch_size must be non-negative")
    base, rem = divmod(batch_size, world)
    start = rank * base + min(rank, rem)
    stop = start + base + (1 if rank < rem else 0)
    return start, stop


def local_roots(global_frontier: torch.Tensor, rank: int, world: int):
    """This rank's roots and the ``batch_offset`` to pass with them."""
    start, stop = partition(int(global_frontier.numel()), rank, world)
    return global_frontier[start:stop].contiguous(), start


def allreduce_gradient(grad: torch.Tensor, group=None) -> torch.Tensor:
    """Sums `grad` over all ranks of `group` in place (NCCL or gloo)."""
    import torch.distributed as dist

    dist.all_reduce(grad, op=dist.ReduceOp.SUM, group=group)
    return grad
