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


# ---------------------------------------------------------------------------
# Row-sharded features (one process per GPU, peers over NVLink)
# ---------------------------------------------------------------------------

def shard_span(num_nodes: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [start, stop) of a `num_nodes`-row table held by `rank`: blocks
    of ceil(num_nodes / world) rows, the last block shorter."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    rows = -(-num_nodes // world) if num_nodes > 0 else 1
    start = min(rank * rows, num_nodes)
    return start, min(start + rows, num_nodes)


def _ipc_share(tensors, group, device: int, stand_in: int):
    """Collective: exports this rank's `tensors` (entries may be None or
    empty) as CUDA IPC handles, gathers every rank's and maps the peers'
    allocations once into `device`'s address space.  Returns, per tensor,
    the list of every rank's pointer valid in this process (`stand_in` for
    a rank's None or empty tensor), and the {handle: base} mappings to close."""
    import ctypes

    import torch.distributed as dist

    from . import _lib

    L = _lib.LIB

    def export(t):
        if t is None or t.numel() == 0:
            return None
        h = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        off = ctypes.c_uint64(0)
        _lib.check(L.fsa_ipc_export(t.data_ptr(), h, ctypes.byref(off)), "fsa_ipc_export")
        return h.raw, off.value

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    shared = [None] * world
    dist.all_gather_object(shared, [export(t) for t in tensors], group=group)
    mapped = {}
    out = [[] for _ in tensors]
    for r, entries in enumerate(shared):
        for k, e in enumerate(entries):
            if r == rank:
                t = tensors[k]
                out[k].append(t.data_ptr() if t is not None and t.numel() > 0 else stand_in)
                continue
            if e is None:
                out[k].append(stand_in)
                continue
            handle, off = e
            if handle not in mapped:
                base = ctypes.c_void_p()
                _lib.check(L.fsa_ipc_open(handle, device, ctypes.byref(base)), "fsa_ipc_open")
                mapped[handle] = base.value
            out[k].append(mapped[handle] + off)
    return out, mapped


class ShardedFeatures:
    """A float32 feature table block-partitioned by row over the ranks of a
    NCCL process group, one GPU per rank, plus its gradient shards.

    Rank r holds rows ``shard_span(num_nodes, r, world)`` in `local` (a
    contiguous [rows, D] tensor on its GPU) and their gradient in `grad`.
    Construction is collective: every rank exports its two shards as CUDA
    IPC handles and maps the others' into its own device's address space, so
    the kernels read remote feature rows and add into remote gradient rows
    directly over NVLink.  Call `close()` on every rank (collective) before
    the process group is destroyed.

    With ``exchange_bytes > 0`` (the same on every rank; see
    `exchange_bytes`) every rank also shares an exchange region of that
    size, and the backward is computed by the owners: each rank publishes
    its saved ids and upstream gradient there, and after a device barrier
    every rank adds the contributions to its own rows from all ranks'
    regions (fsa_sample_agg_2hop_backward_sharded_pull) instead of sending
    one red.add per remote contribution.  Every backward's batch must then
    fit the region on every rank.  With ``persistent=True`` as well, `grad`
    is kept across steps: each backward lists the rows it added into, and
    the next forward zeroes only those (inside its sampling kernel) instead
    of zero-filling the shard; after every backward `grad` still holds
    exactly that step's gradient.
    """

    def __init__(self, local: torch.Tensor, num_nodes: int, group=None, exchange_bytes: int = 0,
                 persistent: bool = False):
        import ctypes

        import torch.distributed as dist

        from . import _lib

        if not local.is_cuda or local.dtype != torch.float32 or local.dim() != 2:
            raise ValueError("local shard must be a 2-D float32 CUDA tensor")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.num_nodes = int(num_nodes)
        start, stop = shard_span(self.num_nodes, self.rank, self.world)
        if local.size(0) != stop - start:
            raise ValueError(f"rank {self.rank} must hold rows [{start}, {stop})")
        if self.world > _lib.MAX_SHARDS:
            raise ValueError(f"at most {_lib.MAX_SHARDS} shards")
        self.start, self.stop = start, stop
        self.shard_rows = -(-self.num_nodes // self.world) if self.num_nodes > 0 else 1
        self.dim = int(local.size(1))
        self.local = local.contiguous()
        self.grad = torch.zeros_like(self.local)
        self.exchange_bytes = int(exchange_bytes)
        if self.exchange_bytes < 0:
            raise ValueError("exchange_bytes must be non-negative")
        self.exchange = (torch.empty((self.exchange_bytes,), dtype=torch.uint8,
                                     device=self.local.device)
                         if self.exchange_bytes > 0 else None)
        # owner-computed backward when there is an exchange region (the same
        # setting on every rank: set it to False on all ranks for the push)
        self.pull = self.exchange is not None
        # with the owner-computed backward: keep `grad` across steps and clear
        # only the rows the previous backward touched (listed by it) instead
        # of zero-filling the shard in every forward
        self.persistent = bool(persistent)
        self._touched = None          # int32 list of local rows (or -1) written by the pull
        self._touched_valid = False   # the list names every row the last backward touched
        self._flag = torch.zeros(1, device=self.local.device)
        self._device = self.local.device.index
        ptrs, self._mapped = _ipc_share(
            [self.local, self.grad, self.exchange], group, self._device, self.local.data_ptr())
        arr = ctypes.c_void_p * self.world
        self.x_ptrs = arr(*ptrs[0])
        self.grad_ptrs = arr(*ptrs[1])
        self.exchange_ptrs = arr(*ptrs[2]) if self.exchange is not None else None

    def device_barrier(self) -> None:
        """Orders the GPUs: the current stream of every rank waits until every
        rank's previously queued work has finished (an NCCL all-reduce of one
        float on the current stream; no host synchronisation)."""
        import torch.distributed as dist

        dist.all_reduce(self._flag, group=self.group)

    def close(self) -> None:
        """Unmaps the peers' shards (collective: call on every rank; no rank
        frees its shards before every rank has unmapped them)."""
        import torch.distributed as dist

        from . import _lib

        torch.cuda.synchronize(self.local.device)
        dist.barrier(group=self.group)
        for base in self._mapped.values():
            _lib.check(_lib.LIB.fsa_ipc_close(base, self._device), "fsa_ipc_close")
        self._mapped.clear()
        self.x_ptrs = self.grad_ptrs = self.exchange_ptrs = None
        dist.barrier(group=self.group)


def exchange_bytes(batch_size: int, fanout1: int, fanout2: int, dim: int) -> int:
    """Exchange-region bytes (`ShardedFeatures(exchange_bytes=...)`) that a
    rank's 2-hop backward of `batch_size` roots needs."""
    from . import _lib

    n = int(_lib.LIB.fsa_exchange_bytes(int(batch_size), int(fanout1), int(fanout2), int(dim)))
    if n == 0:
        raise ValueError("invalid batch size, fanouts or feature dimension")
    return n


def _backward_pull(feats: ShardedFeatures, g, s1, s2):
    """Owner-computes backward: publish this rank's ids and upstream
    gradient, wait for every rank's, add the contributions to this rank's
    rows from all regions."""
    from . import _lib, _stream_handle

    L = _lib.LIB
    B, D = g.shape
    k1, k2 = s1.size(1), s2.size(2)
    need = int(L.fsa_exchange_bytes(B, k1, k2, D))
    if need == 0 or need > feats.exchange_bytes:
        raise RuntimeError(f"a backward of {B} roots at fanouts ({k1}, {k2}) needs an exchange "
                           f"region of {need} bytes; this ShardedFeatures has "
                           f"{feats.exchange_bytes}")
    stream = _stream_handle(g.device)
    touched, capacity = None, 0
    if feats.persistent:
        # one entry per (region, record, slot, position) the pull can visit
        per_root = int(L.fsa_exchange_bytes(1, k1, k2, D)) - 256
        capacity = max((feats.exchange_bytes - 256) // per_root, 0) * feats.world * k1 * k2
        if feats._touched is None or feats._touched.numel() < capacity:
            feats._touched = torch.full((max(capacity, 1),), -1, dtype=torch.int32,
                                        device=g.device)
        touched = feats._touched
    _lib.check(L.fsa_sharded_publish_2hop(feats.exchange.data_ptr(), feats.exchange_bytes,
                                          g.data_ptr(), s1.data_ptr(), s2.data_ptr(), B, D, k1,
                                          k2, stream), "fsa_sharded_publish_2hop")
    # every rank's region holds this step's records
    feats.device_barrier()
    _lib.check(L.fsa_sample_agg_2hop_backward_sharded_pull(
        feats.exchange_ptrs, feats.exchange_bytes, feats.world, feats.rank, feats.grad.data_ptr(),
        feats.shard_rows, feats.num_nodes, D, k1, k2,
        touched.data_ptr() if touched is not None else None, capacity, stream),
        "fsa_sample_agg_2hop_backward_sharded_pull")
    feats._touched_valid = touched is not None


def _forward_2hop_sharded(rowptr, col, feats: ShardedFeatures, frontier, fanout1, fanout2,
                          seed, capture, batch_offset, zero, clear_rows=None):
    from . import _as_int64, _as_seed, _check_fanout_2hop, _check_offset, _DeviceGuard
    from . import _lib, _ptr, _stream_handle

    L = _lib.LIB
    for t, name in ((rowptr, "rowptr"), (col, "col"), (frontier, "frontier")):
        if not t.is_cuda or t.dtype != torch.int32 or t.device != feats.local.device:
            raise RuntimeError(f"{name} must be an int32 tensor on the shard's device")
    if rowptr.numel() != feats.num_nodes + 1:
        raise RuntimeError("rowptr size must be num_nodes + 1")
    fanout1 = _as_int64(fanout1, "fanout1")
    fanout2 = _as_int64(fanout2, "fanout2")
    _check_fanout_2hop(fanout1, fanout2)
    seed = _as_seed(seed)
    off = _check_offset(batch_offset)
    B, D, dev = frontier.size(0), feats.dim, feats.local.device
    with _DeviceGuard(dev):
        if B == 0 or fanout1 == 0 or fanout2 == 0:
            out = torch.zeros((B, D), dtype=torch.float32, device=dev)
            s1 = torch.full((B, fanout1), -1, dtype=torch.int32, device=dev)
            s2 = torch.full((B, fanout1, fanout2), -1, dtype=torch.int32, device=dev)
            if zero is not None:
                zero.zero_()
            if clear_rows is not None:
                _lib.check(L.fsa_zero_rows_f32(feats.grad.data_ptr(), feats.grad.size(0), D,
                                               clear_rows.data_ptr(), clear_rows.numel(),
                                               _stream_handle(dev)), "fsa_zero_rows_f32")
            return out, s1, s2
        out = torch.empty((B, D), dtype=torch.float32, device=dev)
        s1 = torch.empty((B, fanout1), dtype=torch.int32, device=dev) if capture else None
        s2 = torch.empty((B, fanout1, fanout2), dtype=torch.int32, device=dev) if capture else None
        ws_bytes = L.fsa_sample_agg_2hop_workspace_size(B, fanout1, fanout2, int(capture),
                                                        int(capture))
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
        if clear_rows is not None:
            # the rows the previous backward touched, zeroed inside the
            # sampling kernel (no dense fill)
            st = L.fsa_sample_agg_2hop_forward_sharded_zero_rows(
                rowptr.data_ptr(), col.data_ptr(), feats.num_nodes, col.numel(), feats.x_ptrs,
                feats.shard_rows, feats.world, D, frontier.data_ptr(), B, off, fanout1, fanout2,
                seed, out.data_ptr(), _ptr(s1), _ptr(s2), ws.data_ptr(), ws_bytes,
                feats.grad.data_ptr(), feats.grad.size(0), clear_rows.data_ptr(),
                clear_rows.numel(), _stream_handle(dev))
            _lib.check(st, "fsa_sample_agg_2hop_forward_sharded_zero_rows")
        else:
            st = L.fsa_sample_agg_2hop_forward_sharded(
                rowptr.data_ptr(), col.data_ptr(), feats.num_nodes, col.numel(), feats.x_ptrs,
                feats.shard_rows, feats.world, D, frontier.data_ptr(), B, off, fanout1, fanout2,
                seed, out.data_ptr(), _ptr(s1), _ptr(s2), ws.data_ptr(), ws_bytes, _ptr(zero),
                zero.numel() if zero is not None else 0, _stream_handle(dev))
            _lib.check(st, "fsa_sample_agg_2hop_forward_sharded")
    return out, s1, s2


class _Sharded2HopFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, local, rowptr, col, frontier, fanout1, fanout2, replay_seed, batch_offset,
                feats):
        capture = local.requires_grad
        pull = feats.pull and feats.exchange is not None
        # persistent shard: clear the rows the last backward touched instead
        # of zero-filling the whole shard (needs that backward's list)
        clear = (feats._touched if capture and pull and feats.persistent
                 and feats._touched_valid else None)
        out, s1, s2 = _forward_2hop_sharded(rowptr.contiguous(), col.contiguous(), feats,
                                            frontier.contiguous(), fanout1, fanout2,
                                            replay_seed, capture, batch_offset,
                                            feats.grad if capture and clear is None else None,
                                            clear)
        if capture:
            if not (feats.pull and feats.exchange is not None):
                # every rank's gradient shard is zero before any rank's
                # backward adds into it (owner-computed, only the owner adds
                # into its shard, in stream order)
                feats.device_barrier()
            ctx.save_for_backward(s1, s2)
        ctx.feats = feats
        ctx.capture = capture
        return out

    @staticmethod
    def backward(ctx, grad_out):
        from . import _DeviceGuard, _lib, _stream_handle

        if ctx.capture:
            feats = ctx.feats
            s1, s2 = ctx.saved_tensors
            g = grad_out.contiguous()
            B, D = g.shape
            with _DeviceGuard(g.device):
                if feats.pull and feats.exchange is not None:
                    _backward_pull(feats, g, s1, s2)
                else:
                    st = _lib.LIB.fsa_sample_agg_2hop_backward_sharded(
                        g.data_ptr(), s1.data_ptr(), s2.data_ptr(), B, D, s1.size(1),
                        s2.size(2), feats.grad_ptrs, feats.shard_rows, feats.world,
                        feats.num_nodes, _stream_handle(g.device))
                    _lib.check(st, "fsa_sample_agg_2hop_backward_sharded")
                    feats._touched_valid = False  # the list no longer names the touched rows
            # every rank's additions into this rank's shard are complete (and,
            # owner-computed, every rank has read the exchange regions before
            # any rank's next backward rewrites its own)
            feats.device_barrier()
        ctx.feats = None
        return (None,) * 9


def fused_sample_agg_2hop_sharded(rowptr, col, feats: ShardedFeatures, frontier, fanout1,
                                  fanout2, replay_seed=1234, batch_offset=0):
    """2-hop fused sample + mean aggregate over row-sharded features.

    Same ids and outputs as ``fused_sample_agg_2hop`` on the whole table
    (with the same `batch_offset`).  When ``feats.local.requires_grad`` the
    forward zeroes ``feats.grad`` and the backward adds this rank's roots'
    feature gradients into the owning ranks' ``feats.grad`` (over NVLink;
    with an exchange region every owner computes its rows' share from all
    ranks' published ids and upstream gradients instead); after the backward, ``feats.grad`` on every rank holds the gradient of its
    rows summed over all ranks' roots.  Collective when training: every rank
    must call forward and backward the same number of times.
    """
    return _Sharded2HopFn.apply(feats.local, rowptr, col, frontier, fanout1, fanout2,
                                replay_seed, batch_offset, feats)


# ---------------------------------------------------------------------------
# Replicated features, gradient summed over the ranks by exchange
# ---------------------------------------------------------------------------

class GradientExchange:
    """Exchange regions for replicated features: the alternative to an NCCL
    all-reduce of the dense N x D feature gradient after every backward.

    Every rank publishes its step's saved ids and upstream gradient in its
    region (mapped into every peer over CUDA IPC); after a device barrier
    every rank adds every rank's contributions into its own zero-filled
    gradient (the owner-computed backward with one shard covering all rows).
    Every rank then holds the gradient of the whole global batch -- the
    all-reduced gradient, up to the order of the fp32 additions -- while
    NVLink carries (W - 1) * B * (4 (f1 + f1 f2) + 4 D) bytes per rank
    instead of the all-reduce's ~2 * 4 N D.  Construction and `close()` are
    collective.

    With ``persistent=True`` the gradient lives in `grad` (one N x D tensor
    for the exchange's lifetime, like `PersistentGradient`): the backward
    adds into it and autograd produces no gradient for x; each backward lists
    the rows it added into and the next forward zeroes only those (inside its
    sampling kernel) instead of zero-filling N x D, so after every backward
    `grad` holds exactly that step's global gradient.
    """

    def __init__(self, num_nodes: int, dim: int, exchange_bytes: int, device=None, group=None,
                 persistent: bool = False):
        import torch.distributed as dist

        from . import _lib

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.MAX_SHARDS:
            raise ValueError(f"at most {_lib.MAX_SHARDS} ranks")
        if num_nodes < 1 or num_nodes > 0x7FFFFFFF or dim < 0 or exchange_bytes < 256:
            raise ValueError("num_nodes must be in [1, 2^31), dim >= 0, exchange_bytes >= 256")
        dev = torch.device("cuda") if device is None else torch.device(device)
        if dev.type != "cuda":
            raise ValueError("the exchange region lives on a CUDA device")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.num_nodes, self.dim, self.exchange_bytes = int(num_nodes), int(dim), int(exchange_bytes)
        self.exchange = torch.empty((self.exchange_bytes,), dtype=torch.uint8, device=dev)
        self.persistent = bool(persistent)
        self.grad = (torch.zeros((self.num_nodes, self.dim), dtype=torch.float32, device=dev)
                     if self.persistent else None)
        self._touched = None
        self._touched_valid = False
        self._flag = torch.zeros(1, device=dev)
        self._device = dev.index
        import ctypes

        ptrs, self._mapped = _ipc_share([self.exchange], group, self._device,
                                        self.exchange.data_ptr())
        self.exchange_ptrs = (ctypes.c_void_p * self.world)(*ptrs[0])

    def device_barrier(self) -> None:
        """NCCL all-reduce of one float on the current stream (no host sync)."""
        import torch.distributed as dist

        dist.all_reduce(self._flag, group=self.group)

    def close(self) -> None:
        """Unmaps the peers' regions (collective)."""
        import torch.distributed as dist

        from . import _lib

        torch.cuda.synchronize(self.exchange.device)
        dist.barrier(group=self.group)
        for base in self._mapped.values():
            _lib.check(_lib.LIB.fsa_ipc_close(base, self._device), "fsa_ipc_close")
        self._mapped.clear()
        self.exchange_ptrs = None
        dist.barrier(group=self.group)


class _Exchange2HopFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, rowptr, col, frontier, fanout1, fanout2, replay_seed, batch_offset, ex):
        from . import _as_int64, _as_seed, _check_fanout_2hop, _check_offset
        from . import _check_python_inputs, _DeviceGuard, _lib, _stream_handle

        L = _lib.LIB
        _check_python_inputs(rowptr, col, x, frontier)
        fanout1 = _as_int64(fanout1, "fanout1")
        fanout2 = _as_int64(fanout2, "fanout2")
        _check_fanout_2hop(fanout1, fanout2)
        seed = _as_seed(replay_seed)
        off = _check_offset(batch_offset)
        rowptr, col, frontier = rowptr.contiguous(), col.contiguous(), frontier.contiguous()
        xc = x.detach().contiguous()
        if xc.dim() != 2 or rowptr.numel() != xc.size(0) + 1:
            raise RuntimeError("x must be [N, D] with rowptr of N + 1 entries")
        N, D = xc.shape
        B = frontier.numel()
        if N != ex.num_nodes or D != ex.dim:
            raise RuntimeError("x must be [num_nodes, dim] of the GradientExchange")
        if xc.device != ex.exchange.device:
            raise RuntimeError("x must be on the GradientExchange's device")
        dev = xc.device
        with _DeviceGuard(dev):
            out = torch.empty((B, D), dtype=torch.float32, device=dev)
            s1 = torch.full((B, fanout1), -1, dtype=torch.int32, device=dev)
            s2 = torch.full((B, fanout1, fanout2), -1, dtype=torch.int32, device=dev)
            ws_bytes = L.fsa_sample_agg_2hop_workspace_size(B, fanout1, fanout2, 1, 1)
            ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
            stream = _stream_handle(dev)
            if ex.persistent and ex.grad is None:  # switched on after construction
                ex.grad = torch.zeros_like(xc)
                ex._touched_valid = False
            if ex.persistent and ex._touched_valid:
                # the rows the previous backward added into, zeroed inside the
                # sampling kernel (no N x D fill)
                grad = ex.grad
                _lib.check(L.fsa_sample_agg_2hop_forward_zero_rows(
                    rowptr.data_ptr(), col.data_ptr(), N, col.numel(), xc.data_ptr(), D,
                    frontier.data_ptr(), B, off, fanout1, fanout2, seed, out.data_ptr(),
                    s1.data_ptr(), s2.data_ptr(), ws.data_ptr(), ws_bytes, grad.data_ptr(),
                    ex._touched.data_ptr(), ex._touched.numel(), stream),
                    "fsa_sample_agg_2hop_forward_zero_rows")
            else:
                grad = ex.grad if ex.persistent else torch.empty_like(xc)
                _lib.check(L.fsa_sample_agg_2hop_forward(
                    rowptr.data_ptr(), col.data_ptr(), N, col.numel(), xc.data_ptr(), D,
                    frontier.data_ptr(), B, off, fanout1, fanout2, seed, out.data_ptr(),
                    s1.data_ptr(), s2.data_ptr(), ws.data_ptr(), ws_bytes, grad.data_ptr(),
                    grad.numel(), stream), "fsa_sample_agg_2hop_forward")
            if fanout1 == 0 or fanout2 == 0:
                out.zero_()  # nothing sampled (fuseop/binding.cpp:183-185)
        ctx.save_for_backward(s1, s2)
        ctx.grad = grad
        ctx.ex = ex
        return out

    @staticmethod
    def backward(ctx, grad_out):
        from . import _DeviceGuard, _lib, _stream_handle

        ex = ctx.ex
        s1, s2 = ctx.saved_tensors
        grad = ctx.grad
        ctx.grad = ctx.ex = None
        g = grad_out.contiguous()
        B, D = g.shape
        k1, k2 = s1.size(1), s2.size(2)
        L = _lib.LIB
        need = int(L.fsa_exchange_bytes(B, k1, k2, D))
        if need == 0 or need > ex.exchange_bytes:
            raise RuntimeError(f"a backward of {B} roots at fanouts ({k1}, {k2}) needs an exchange "
                               f"region of {need} bytes; this GradientExchange has "
                               f"{ex.exchange_bytes}")
        with _DeviceGuard(g.device):
            stream = _stream_handle(g.device)
            _lib.check(L.fsa_sharded_publish_2hop(ex.exchange.data_ptr(), ex.exchange_bytes,
                                                  g.data_ptr(), s1.data_ptr(), s2.data_ptr(), B,
                                                  D, k1, k2, stream), "fsa_sharded_publish_2hop")
            ex.device_barrier()  # every rank's region holds this step's records
            touched, capacity = None, 0
            if ex.persistent:
                per_root = int(L.fsa_exchange_bytes(1, k1, k2, D)) - 256
                capacity = max((ex.exchange_bytes - 256) // per_root, 0) * ex.world * k1 * k2
                if ex._touched is None or ex._touched.numel() < capacity:
                    ex._touched = torch.full((max(capacity, 1),), -1, dtype=torch.int32,
                                             device=g.device)
                touched = ex._touched
            # one shard of all N rows: every contribution of every rank is this rank's
            _lib.check(L.fsa_sample_agg_2hop_backward_sharded_pull(
                ex.exchange_ptrs, ex.exchange_bytes, ex.world, 0, grad.data_ptr(), ex.num_nodes,
                ex.num_nodes, D, k1, k2, touched.data_ptr() if touched is not None else None,
                capacity, stream), "fsa_sample_agg_2hop_backward_sharded_pull")
            ex._touched_valid = touched is not None
            ex.device_barrier()  # every rank has read the regions before they are rewritten
        if ex.persistent:
            return (None,) * 9  # the gradient is in ex.grad
        return (grad,) + (None,) * 8


def fused_sample_agg_2hop_exchange(rowptr, col, x, frontier, fanout1, fanout2,
                                   replay_seed=1234, batch_offset=0, *, exchange):
    """``fused_sample_agg_2hop`` on replicated features whose backward gives
    every rank the feature gradient of the whole global batch (what an
    all-reduce of the per-rank gradients gives) through `exchange`, a
    `GradientExchange`.  The ids and outputs are those of
    ``fused_sample_agg_2hop`` with the same `batch_offset`.  Collective
    when training: every rank calls forward and backward together.  Without
    ``x.requires_grad`` this is the plain op."""
    from . import fused_sample_agg_2hop

    if not x.requires_grad:
        return fused_sample_agg_2hop(rowptr, col, x, frontier, fanout1, fanout2, replay_seed,
                                     batch_offset=batch_offset)
    return _Exchange2HopFn.apply(x, rowptr, col, frontier, fanout1, fanout2, replay_seed,
                                 batch_offset, exchange)
