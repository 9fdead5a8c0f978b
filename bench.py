"""Benchmark: 2-hop fused sample + mean aggregate, forward + backward, roots/s.

Workload (default ``c2_2hop_powerlaw``): symmetric Chung-Lu power-law CSR,
N = 2.45M nodes, ~123M directed int32 edges (exponent 2.1, degree cap
20,000), fp32 features 2.45M x 100 (trainable), fanouts (15, 10), 1024
distinct uniform roots per GPU per step, root batches / replay seeds 0..99
used round-robin.  Inputs are synthetic (seeded) stand-ins for the
reference's public datasets.

A step is one batch through the public API: ``x.grad = None``,
``out = fused_sample_agg_2hop(...)`` with x requiring grad (saved-index
capture), ``out.backward(grad_out)`` -- i.e. the dense N x D gradient zero
fill, the fused sample + gather kernel and the replay scatter kernel.

Timing: W untimed warm-up steps, then exactly K steps bracketed by a
barrier + cuda synchronize, CUDA events on the launching stream, max over
ranks.  x (980 MB) is gathered at random and the 980 MB gradient is
rewritten every step, so inputs exceed the 126 MB L2 between steps.

Multi-GPU (torchrun): one process per GPU, graph and features replicated,
each rank takes its contiguous 1024-root slice of a global batch with
``batch_offset = rank * 1024`` (ids identical to a single-GPU run of the
global batch); no collective on the data path (weak scaling).  After the
main measurement, on 2+ GPUs: the same step followed by the NCCL all-reduce
of the dense feature gradient (`replicated_allreduce`), the same gradient
summed through exchange regions instead (`replicated_exchange`), the
row-sharded mode checked bit for bit against the replicated op and timed
(`sharded`), and the 100M-node configuration (`c5`; replicated on one GPU,
row-sharded on 2+).

``--impl reference`` runs the reference's own CUDA op (built from its
sources into oracle/_ref) on the same workload through its public API, on
every rank (each rank times its own 1024 roots).  The CPU baseline (rank 0,
N=1) is the sequential C oracle on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import datetime
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))


def _load_by_path(name: str, path: Path):
    """Imports one module file without importing the package around it:
    `fusesampleagg_b200/__init__.py` loads the library's .so files, which the
    reference arm must not map."""
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod  # dataclasses look their module up while it executes
    spec.loader.exec_module(mod)
    return mod


synthetic = _load_by_path("_fsa_bench_synthetic", REPO / "fusesampleagg_b200" / "synthetic.py")

METRIC = "2-hop fwd+bwd roots/s"
PEAKS_PATH = REPO / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
NOMINAL_HBM_GBS = 8000.0

# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum, in
# bytes) that ncu measured for each kernel of a workload, from the captures
# summarised in profiles/ (commands there).  The draw kernel with the fused
# fill writes 919 MB of the 980 MB fill during its own launch; the rest
# leaves L2 as dirty lines during the next kernels.
NCU_TRAFFIC = {
    "c2_2hop_powerlaw": {
        "draw": 1.09e6 + 919.0e6,
        "gather": 55.53e6 + 0.62e6,
        "plan": 1.88e6,
        "scan": 0.02e6,
        "bwd": 42.32e6 + 3.25e6,
    },
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# The process's stdout carries exactly one JSON line.  Libraries write to
# file descriptor 1 on their own (NCCL's version banner, for one), so main()
# points descriptor 1 at stderr and the result goes to a saved copy of the
# original stdout.
_RESULT_FD = None


def emit(obj) -> None:
    data = json.dumps(obj) + "\n"
    if _RESULT_FD is None:
        sys.stdout.write(data)
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, data.encode())


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------

class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False

    def init(self):
        if self.world > 1 and not self.pg:
            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local_rank))
            self.pg = True

    def barrier(self):
        if self.pg:
            import torch.distributed as dist

            dist.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            import torch.distributed as dist

            dist.destroy_process_group()
            self.pg = False


# ---------------------------------------------------------------------------
# Clock sampling (NVML through nvidia-smi) during the timed region
# ---------------------------------------------------------------------------

CLOCK_FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.window = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="fsa_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def mark(self, t0: float, t1: float):
        self.window = (t0, t1)

    def stop(self) -> dict:
        if self.proc is None:
            return {"error": "nvidia-smi unavailable"}
        time.sleep(0.12)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return {"error": "no samples"}
        inside = [r for r in rows if self.window and self.window[0] <= r[0] <= self.window[1]]
        window = "timed"
        if not inside:
            inside, window = rows, "warmup+timed (timed region shorter than the sample period)"
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[k] for r in inside for k in range(4) if r[3][k] == "Active"})
        return {
            "sm_mhz": statistics.median(r[1] for r in inside),
            "sm_max_mhz": max(r[2] for r in inside),
            "reasons": reasons,
            "samples": len(inside),
            "window": window,
        }


# ---------------------------------------------------------------------------
# Workload
# ---------------------------------------------------------------------------

def load_peaks() -> tuple[float, str]:
    try:
        peaks = json.loads(PEAKS_PATH.read_text())
        return float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


class Inputs:
    def __init__(self, w: synthetic.Workload, dev: torch.device, rank: int, world: int,
                 batches: int):
        t0 = time.time()
        g = w.graph(seed=0, device=dev)
        self.rowptr, self.col = g.rowptr, g.col
        self.stats = synthetic.degree_stats(g)
        del g
        self.n = self.rowptr.numel() - 1
        self.x = w.features(seed=1, device=dev).requires_grad_(True)
        self.B = w.batch
        self.offset = rank * w.batch
        self.frontiers = []
        for s in range(batches):
            full = synthetic.root_batch(self.n, w.batch * world, seed=s, device=dev)
            self.frontiers.append(full[self.offset:self.offset + w.batch].contiguous())
        self.seeds = list(range(batches))
        self.grad_out = synthetic.features(w.batch, w.dim, seed=2, device=dev)
        torch.cuda.synchronize()
        torch.cuda.empty_cache()  # drop the graph generator's temporaries
        self.setup_s = time.time() - t0


def graph_identical_across_ranks(inp: Inputs, dist: Dist) -> bool | None:
    """Whether every rank generated the same CSR (None on one GPU): an exact
    position-weighted int64 sum of rowptr and col (wrapping, so independent
    of summation order), compared by an all-reduce of its min and max."""
    if not dist.pg:
        return None
    import torch.distributed as tdist

    fp = torch.zeros(2, dtype=torch.int64, device=inp.rowptr.device)
    for k, t in enumerate((inp.rowptr, inp.col)):
        step = 1 << 27
        for s in range(0, t.numel(), step):
            part = t[s:s + step].to(torch.int64)
            wgt = torch.arange(s, s + part.numel(), device=part.device) % 1021 + 1
            fp[k] += (part * wgt).sum()
    lo, hi = fp.clone(), fp.clone()
    tdist.all_reduce(lo, op=tdist.ReduceOp.MIN)
    tdist.all_reduce(hi, op=tdist.ReduceOp.MAX)
    return bool(torch.equal(lo, hi))


def byte_model(w, inp: Inputs, batches: list[int]) -> dict:
    """Algorithmic bytes per batch, per kernel, averaged over `batches`, from
    the samples the op itself draws (independent of the implementation).

    plan   = 4B (frontier) + 8(B + valid middles) (rowptr pairs) + 4 take1
             (first-hop col ids) + 4 B k1 (saved first-hop ids)
    draw   = 24 B k1 (second-hop row table: state, take, draws, prefix)
             + 4 N D (the fused dense-gradient zero fill)
    gather = 4 valid leaves (col ids) + 4 D valid leaves (feature rows)
             + 4 D B (out) + 4 B k1 k2 (saved second-hop ids)
    bwd    = 4 D B (grad_out) + saved ids + 8 D valid leaves (atomic RMW)
    """
    import fusesampleagg_b200 as fsa

    k1, k2 = w.fanouts
    B, D = inp.B, w.dim
    keys = ("plan", "draw", "gather", "bwd", "unique_leaf_rows", "valid_leaves", "rng_draws")
    tot = {k: 0.0 for k in keys}
    deg = (inp.rowptr[1:] - inp.rowptr[:-1]).long()
    with torch.no_grad():
        for i in batches:
            _, s1, s2 = fsa.fused_sample_agg_2hop_with_samples(
                inp.rowptr, inp.col, inp.x.detach(), inp.frontiers[i], k1, k2,
                replay_seed=inp.seeds[i], batch_offset=inp.offset)
            valid_mid = int((s1 >= 0).sum())
            valid_leaves = int((s2 >= 0).sum())
            saved1, saved2 = 4 * B * k1, 4 * B * k1 * k2
            tot["plan"] += 4 * B + 8 * (B + valid_mid) + 4 * valid_mid + saved1
            tot["draw"] += 24 * B * k1 + 4.0 * inp.n * D
            tot["gather"] += 4 * valid_leaves + 4 * D * valid_leaves + 4 * D * B + saved2
            tot["bwd"] += 4 * D * B + saved1 + saved2 + 8 * D * valid_leaves
            # Reservoir draws (one xorshift64* output each) past the first
            # `fanout` positions of every sampled row: the sampler's work.
            mids = s1[s1 >= 0].long()
            tot["rng_draws"] += float((deg[inp.frontiers[i].long()] - k1).clamp_min(0).sum()
                                      + (deg[mids] - k2).clamp_min(0).sum())
            leaves = s2[s2 >= 0]
            tot["valid_leaves"] += valid_leaves
            tot["unique_leaf_rows"] += int(torch.unique(leaves).numel())
    n = max(len(batches), 1)
    out = {k: v / n for k, v in tot.items()}
    out["scan"] = 16.0 * B  # root counts in, prefix out
    out["fill"] = 4.0 * inp.n * D
    return out


# ---------------------------------------------------------------------------
# Steps
# ---------------------------------------------------------------------------

def make_step(api, w, inp: Inputs, batch_offset: bool):
    k1, k2 = w.fanouts
    nb = len(inp.frontiers)
    kw = {"batch_offset": inp.offset} if batch_offset else {}

    def step(i, ev=None):
        j = i % nb
        inp.x.grad = None
        if ev is not None:
            ev[0].record()
        out = api.fused_sample_agg_2hop(inp.rowptr, inp.col, inp.x, inp.frontiers[j], k1, k2,
                                        replay_seed=inp.seeds[j], **kw)
        if ev is not None:
            ev[1].record()
        out.backward(inp.grad_out)
        if ev is not None:
            ev[2].record()
        return out

    return step


def make_e2e_step(api, w, inp: Inputs, batch_offset: bool):
    """Public-API step with host buffers: every step copies its roots and
    upstream gradient from pinned host memory (one packed buffer per root
    batch, one copy) and reads its output back into pinned memory, where the
    host reads it.  As a data loader would, the copies run on a second
    stream: step i+1's inputs are copied while step i computes (double
    buffered), and step i's output is read back while step i+1 computes; the
    host reads step i's output at the start of step i+2 (waiting for its
    copy), which also bounds how far the host runs ahead of the GPU.
    `reset()` drops the prefetched inputs, so the first step after it copies
    its own inputs first."""
    k1, k2 = w.fanouts
    nb = len(inp.frontiers)
    kw = {"batch_offset": inp.offset} if batch_offset else {}
    dev = inp.x.device
    fr_bytes = inp.frontiers[0].numel() * 4
    go_bytes = inp.grad_out.numel() * 4
    nbytes = fr_bytes + go_bytes
    go_u8 = inp.grad_out.reshape(-1).view(torch.uint8).cpu()
    host_in = []
    for f in inp.frontiers:
        h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        h[:fr_bytes].copy_(f.cpu().view(torch.uint8))
        h[fr_bytes:].copy_(go_u8)
        host_in.append(h)
    host_out = [torch.empty((w.batch, w.dim), dtype=torch.float32).pin_memory() for _ in range(2)]
    dev_in = [torch.empty(nbytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    dev_fr = [b[:fr_bytes].view(torch.int32) for b in dev_in]
    dev_go = [b[fr_bytes:].view(torch.float32).view(w.batch, w.dim) for b in dev_in]
    # Setup (untimed): move every pinned buffer through the DMA path once, as
    # a data loader's first epoch would; the first copy out of a freshly
    # pinned buffer costs far more than later ones.
    for h in host_in:
        dev_in[0].copy_(h, non_blocking=True)
    for h in host_out:
        h.copy_(dev_in[0][: h.numel() * 4].view(torch.float32).view_as(h), non_blocking=True)
    torch.cuda.synchronize(dev)
    comp = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(device=dev)
    free = [None, None]       # event after the last compute that read a slot
    ready = {}                # step -> event of its input copy
    d2h = host_out[0].numel() * 4
    # Events are reused two steps later: by then every wait on their previous
    # record has been enqueued (a wait binds to the record it sees).
    ready_ev = [torch.cuda.Event() for _ in range(2)]
    done_ev = [torch.cuda.Event() for _ in range(2)]
    out_ev = [torch.cuda.Event() for _ in range(2)]
    pending = [False, False]  # an output copy into host_out[slot] not read yet
    checksum = [0.0]

    def copy_inputs(i):
        # on the copy stream
        slot = i % 2
        if free[slot] is not None:
            copy.wait_event(free[slot])
        dev_in[slot].copy_(host_in[i % nb], non_blocking=True)
        ev = ready_ev[slot]
        ev.record(copy)
        ready[i] = ev

    def step(i):
        slot = i % 2
        if pending[slot]:
            # the host reads step i-2's result before its buffer is reused
            out_ev[slot].synchronize()
            checksum[0] += float(host_out[slot][0, 0])
            pending[slot] = False
        if i not in ready:
            torch.cuda.set_stream(copy)
            copy_inputs(i)
            torch.cuda.set_stream(comp)
        comp.wait_event(ready.pop(i))
        inp.x.grad = None
        out = api.fused_sample_agg_2hop(inp.rowptr, inp.col, inp.x, dev_fr[slot], k1, k2,
                                        replay_seed=inp.seeds[i % nb], **kw)
        out.backward(dev_go[slot])
        done = done_ev[slot]
        done.record(comp)
        free[slot] = done
        torch.cuda.set_stream(copy)
        copy_inputs(i + 1)              # does not wait for this step's compute
        copy.wait_event(done)
        host_out[slot].copy_(out.detach(), non_blocking=True)
        out_ev[slot].record(copy)
        torch.cuda.set_stream(comp)
        pending[slot] = True
        out.record_stream(copy)

    step.reset = ready.clear
    # the last output read-back belongs to the timed region
    step.drain = lambda: comp.wait_stream(copy)
    return step, nbytes, d2h


def with_gradient_allreduce(step, inp: Inputs):
    """The step followed by the replicated mode's optional collective: an
    NCCL all-reduce (sum) of the dense feature gradient over the ranks, on the
    compute stream (`sharding.allreduce_gradient`)."""
    from fusesampleagg_b200.sharding import allreduce_gradient

    def run_step(i, *a):
        out = step(i, *a)
        allreduce_gradient(inp.x.grad)
        return out

    for attr in ("reset", "drain"):
        if hasattr(step, attr):
            setattr(run_step, attr, getattr(step, attr))
    return run_step


def timed(step, steps: int, warmup: int, dist: Dist, sampler=None, phase_events=False):
    for i in range(warmup):
        step(i)
    if hasattr(step, "reset"):
        step.reset()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    evs = None
    if phase_events:
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    start.record()
    for i in range(steps):
        if evs is not None:
            step(warmup + i, evs[i])
        else:
            step(warmup + i)
    if hasattr(step, "drain"):
        step.drain()
    end.record()
    torch.cuda.synchronize()
    t_wall1 = time.time()
    dist.barrier()
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.mark(t_wall0, t_wall1)
    ms = start.elapsed_time(end)
    phases = None
    if evs is not None:
        fwd = sum(e[0].elapsed_time(e[1]) for e in evs) / steps
        bwd = sum(e[1].elapsed_time(e[2]) for e in evs) / steps
        phases = {"forward_ms": fwd, "backward_ms": bwd}
    return dist.max(ms), phases


def kernel_times(w, inp: Inputs, iters: int) -> dict:
    """Per-kernel CUDA-event durations (us) through the C ABI on the current
    stream, same inputs as the timed steps.  The step's own configuration
    first: the 2-hop forward with the dense-gradient zero fill fused into its
    draw kernel, timed per kernel with the library's phase events, then the
    backward.  For comparison: the forward without the fill and the
    stand-alone fill kernel."""
    from fusesampleagg_b200 import _lib

    L = _lib.LIB
    k1, k2 = w.fanouts
    B, D, n = inp.B, w.dim, inp.n
    dev = inp.x.device
    out = torch.empty((B, D), device=dev)
    s1 = torch.empty((B, k1), dtype=torch.int32, device=dev)
    s2 = torch.empty((B, k1, k2), dtype=torch.int32, device=dev)
    grad = torch.empty((n, D), device=dev)
    ws_bytes = L.fsa_sample_agg_2hop_workspace_size(B, k1, k2, 1, 1)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    x = inp.x.detach()

    def fwd(j, fill):
        _lib.check(L.fsa_sample_agg_2hop_forward(
            inp.rowptr.data_ptr(), inp.col.data_ptr(), n, inp.col.numel(), x.data_ptr(), D,
            inp.frontiers[j].data_ptr(), B, inp.offset, k1, k2, inp.seeds[j], out.data_ptr(),
            s1.data_ptr(), s2.data_ptr(), ws.data_ptr(), ws_bytes,
            grad.data_ptr() if fill else None, grad.numel() if fill else 0, stream), "fwd")

    def bwd():
        _lib.check(L.fsa_sample_agg_2hop_backward(
            inp.grad_out.data_ptr(), s1.data_ptr(), s2.data_ptr(), B, D, k1, k2,
            grad.data_ptr(), n, stream), "bwd")

    nb = len(inp.frontiers)
    for it in range(3):
        fwd(it % nb, True)
        bwd()
    torch.cuda.synchronize()
    res = {"bwd": 0.0, "bwd_sorted": 0.0, "fwd_nofill": 0.0, "fill_alone": 0.0}
    sws_bytes = L.fsa_sample_agg_2hop_backward_sorted_workspace_size(n, B, k1, k2)
    sws = torch.empty((sws_bytes,), dtype=torch.uint8, device=dev)

    def bwd_sorted():
        _lib.check(L.fsa_sample_agg_2hop_backward_sorted(
            inp.grad_out.data_ptr(), s1.data_ptr(), s2.data_ptr(), B, D, k1, k2,
            grad.data_ptr(), n, sws.data_ptr(), sws_bytes, stream), "bwd_sorted")

    bwd_sorted()
    _lib.phase_timing(True)
    try:
        for it in range(iters):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            fwd(it % nb, True)
            ev[0].record()
            bwd()
            ev[1].record()
            torch.cuda.synchronize()
            res["bwd"] += ev[0].elapsed_time(ev[1])
        phases, calls = _lib.phase_times()
    finally:
        _lib.phase_timing(False)
    for it in range(iters):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        fwd(it % nb, True)
        ev[0].record()
        bwd_sorted()
        ev[1].record()
        torch.cuda.synchronize()
        res["bwd_sorted"] += ev[0].elapsed_time(ev[1])
    del sws
    for it in range(iters):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        _lib.check(L.fsa_fill_zero_f32(grad.data_ptr(), grad.numel(), stream), "fill")
        ev[1].record()
        fwd(it % nb, False)
        ev[2].record()
        torch.cuda.synchronize()
        res["fill_alone"] += ev[0].elapsed_time(ev[1])
        res["fwd_nofill"] += ev[1].elapsed_time(ev[2])
    # The backward after a forward without the fused fill (no dirty fill
    # lines draining from L2 while it runs), and the row clear of the
    # persistent gradient (the rows of one step's saved ids) launched
    # back to back, so that no host gap falls between the events.
    res["bwd_after_nofill"] = 0.0
    for it in range(iters):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        fwd(it % nb, False)
        ev[0].record()
        bwd()
        ev[1].record()
        torch.cuda.synchronize()
        res["bwd_after_nofill"] += ev[0].elapsed_time(ev[1])
    # The backward after the forward and a 256 MB read, which writes the
    # dirty lines the forward left in L2 back to HBM before the backward
    # starts; against "bwd", the share of the backward's live time that is
    # the forward's write-back.
    res["bwd_after_writeback"] = 0.0
    flush = torch.ones(64 << 20, device=dev)
    acc = torch.zeros(1, device=dev)
    for it in range(iters):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        fwd(it % nb, True)
        torch.sum(flush, dim=0, keepdim=True, out=acc)
        ev[0].record()
        bwd()
        ev[1].record()
        torch.cuda.synchronize()
        res["bwd_after_writeback"] += ev[0].elapsed_time(ev[1])
    del flush, acc
    reps = 20
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    fwd(0, False)
    ev[0].record()
    for _ in range(reps):
        _lib.check(L.fsa_zero_rows_f32(grad.data_ptr(), n, D, s2.data_ptr(), s2.numel(), stream),
                   "zero rows")
    ev[1].record()
    torch.cuda.synchronize()
    res["zero_rows"] = ev[0].elapsed_time(ev[1]) * iters / reps
    times = {k: 1000.0 * v / calls for k, v in phases.items()}
    times.update({k: 1000.0 * v / iters for k, v in res.items()})
    return times


# ---------------------------------------------------------------------------
# CPU baseline (oracle on the host cores)
# ---------------------------------------------------------------------------

def cpu_baseline(w, inp: Inputs, budget_s: float = 12.0) -> dict:
    from oracle import oracle

    threads = os.cpu_count() or 1
    rowptr = inp.rowptr.cpu().numpy()
    col = inp.col.cpu().numpy()
    x = inp.x.detach().cpu().numpy()
    go = inp.grad_out.cpu().numpy()
    k1, k2 = w.fanouts
    done = 0
    t0 = time.time()
    batches = 0
    while time.time() - t0 < budget_s and batches < len(inp.frontiers):
        fr = inp.frontiers[batches].cpu().numpy()
        s1, s2 = oracle.sample_2hop(rowptr, col, fr, k1, k2, inp.seeds[batches],
                                    batch_offset=inp.offset, threads=threads)
        oracle.forward_2hop(x, s2, threads=threads)
        oracle.backward_2hop(go, s1, s2, inp.n)  # allocates + zero-fills N x D
        done += fr.shape[0]
        batches += 1
    dt = time.time() - t0
    return {
        "value": done / dt,
        "unit": "roots/s",
        "cores": threads,
        "kind": "port",
        "sample": (f"{batches} batches x {inp.B} roots of the same workload through the C oracle "
                   f"(sampling and forward on {threads} OpenMP threads, backward incl. the dense "
                   f"N x D gradient zero-fill on 1 thread), {dt:.1f} s"),
    }


# ---------------------------------------------------------------------------
# Arms
# ---------------------------------------------------------------------------

def sharded_api(inp: Inputs, w):
    """The package's API with the features row-sharded over the ranks: this
    rank keeps only its rows, the others' are mapped over NVLink.  Returns an
    object with the `fused_sample_agg_2hop` / `launch_count` calls the steps
    use (its x argument is ignored) and the ShardedFeatures."""
    import fusesampleagg_b200 as fsa
    from fusesampleagg_b200 import sharding

    start, stop = sharding.shard_span(inp.n, int(os.environ.get("RANK", "0")),
                                      int(os.environ.get("WORLD_SIZE", "1")))
    local = inp.x.detach()[start:stop].clone().requires_grad_(True)
    k1, k2 = w.fanouts
    feats = sharding.ShardedFeatures(local, inp.n,
                                     exchange_bytes=sharding.exchange_bytes(w.batch, k1, k2, w.dim))
    # the whole table is not needed any more: keep a 1-row stand-in so that
    # the steps' `x.grad = None` still works
    inp.x = torch.zeros((1, w.dim), device=local.device, requires_grad=True)
    torch.cuda.empty_cache()

    class Api:
        @staticmethod
        def fused_sample_agg_2hop(rowptr, col, x, frontier, k1, k2, replay_seed=1234,
                                  batch_offset=0):
            return sharding.fused_sample_agg_2hop_sharded(rowptr, col, feats, frontier, k1, k2,
                                                          replay_seed, batch_offset)

        launch_count = staticmethod(fsa.launch_count)

    return Api, feats


def mapped_repo_libraries() -> list[str]:
    """Shared objects under this repository mapped into this process
    (/proc/self/maps), as paths relative to the repository."""
    found = set()
    try:
        with open("/proc/self/maps") as fh:
            for line in fh:
                parts = line.split()
                if len(parts) >= 6 and ".so" in parts[-1]:
                    p = Path(parts[-1])
                    if p.is_relative_to(REPO):
                        found.add(str(p.relative_to(REPO)))
    except OSError:
        pass
    return sorted(found)


def check_reference_arm_libraries() -> list[str]:
    """The reference arm may map the reference op's own extension and nothing
    else built in this repository."""
    libs = mapped_repo_libraries()
    foreign = [p for p in libs if not p.startswith("oracle/_ref/fuseop/")]
    if foreign:
        raise SystemExit(f"reference arm mapped this repository's libraries: {foreign}")
    return libs


def persistent_leg(w, inp: Inputs, args, dist: Dist, check: bool = True, steps: int | None = None,
                   warmup: int | None = None) -> dict:
    """The opt-in persistent gradient (``grad_buffer=PersistentGradient``):
    the same steps, but each step's forward clears only the rows the previous
    step's backward touched (``clear_grad_buffer=True``: zeroed inside the
    sampling kernel from the previous step's saved ids) and the backward adds
    into the caller's buffer, instead of a fresh dense N x D gradient
    zero-filled every step.  Device-timed like the main measurement; then one
    step's buffer is compared with the default path's gradient of the same
    batch (rtol 1e-5 / atol 1e-6), and the forward and backward are timed
    with events."""
    import fusesampleagg_b200 as fsa

    k1, k2 = w.fanouts
    nb = len(inp.frontiers)
    buf = fsa.PersistentGradient(inp.x)

    def step(i, ev=None):
        j = i % nb
        if ev is not None:
            ev[0].record()
        out = fsa.fused_sample_agg_2hop(inp.rowptr, inp.col, inp.x, inp.frontiers[j], k1, k2,
                                        replay_seed=inp.seeds[j], batch_offset=inp.offset,
                                        grad_buffer=buf, clear_grad_buffer=True)
        if ev is not None:
            ev[1].record()
        out.backward(inp.grad_out)
        if ev is not None:
            ev[2].record()

    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    launches0 = fsa.launch_count()
    ms, phases = timed(step, steps, warmup, dist, phase_events=True)
    ms, _ = timed(step, steps, warmup, dist)
    launches = (fsa.launch_count() - launches0) * steps // (2 * (steps + warmup))
    rows = sum(int((ids >= 0).sum()) for ids, _ in buf._touched)
    ok = None
    if check:
        # equality with the default path on one batch
        j = (warmup + steps) % nb
        fsa.fused_sample_agg_2hop(inp.rowptr, inp.col, inp.x, inp.frontiers[j], k1, k2,
                                  replay_seed=inp.seeds[j], batch_offset=inp.offset,
                                  grad_buffer=buf, clear_grad_buffer=True).backward(inp.grad_out)
        inp.x.grad = None
        fsa.fused_sample_agg_2hop(inp.rowptr, inp.col, inp.x, inp.frontiers[j], k1, k2,
                                  replay_seed=inp.seeds[j], batch_offset=inp.offset
                                  ).backward(inp.grad_out)
        torch.cuda.synchronize()
        ok = bool(torch.isclose(buf.grad, inp.x.grad, rtol=1e-5, atol=1e-6).all())
        inp.x.grad = None
    del buf
    torch.cuda.empty_cache()
    units = w.batch * dist.world * steps
    return {
        "value": units / (ms / 1000.0),
        "unit": "roots/s",
        "ms_per_step": ms / steps,
        "steps": steps,
        "warmup": warmup,
        "gpu_launches": launches,
        "phases_ms": phases,
        "rows_cleared_per_step": rows,
        "clear": ("rows of the previous step's saved ids zeroed by the draw kernel's two "
                  "fill warps (fsa_sample_agg_2hop_forward_zero_rows), no kernel of its own"),
        "matches_fresh_gradient": ok,
        "check": ("one step's buffer vs the default path's dense gradient of the same batch, "
                  "rtol 1e-5 / atol 1e-6" if check else
                  "not repeated here (two more N x D tensors); checked on C2 and in the tests"),
        "api": "fused_sample_agg_2hop(..., grad_buffer=PersistentGradient(x), "
               "clear_grad_buffer=True)",
    }


def allreduce_leg(w, inp: Inputs, args, dist: Dist, base_ms_per_step: float) -> dict:
    """The replicated mode's data-parallel training step (2+ GPUs): the
    same timed step followed by an NCCL all-reduce (sum) of the dense N x D
    feature gradient over the ranks, so that every rank holds the gradient of
    the whole global batch.  Device-timed, max over ranks."""
    import fusesampleagg_b200 as fsa

    launches0 = fsa.launch_count()
    step = with_gradient_allreduce(make_step(fsa, w, inp, batch_offset=True), inp)
    ms, _ = timed(step, args.steps, args.warmup, dist)
    launches = (fsa.launch_count() - launches0) * args.steps // (args.steps + args.warmup)
    units = w.batch * dist.world * args.steps
    grad_bytes = 4 * inp.x.numel()
    per_step = ms / args.steps
    ar_ms = max(per_step - base_ms_per_step, 0.0)
    return {
        "value": units / (ms / 1000.0),
        "unit": "roots/s",
        "ms_per_step": per_step,
        "steps": args.steps,
        "warmup": args.warmup,
        "gpu_launches": launches,
        "allreduce_bytes": grad_bytes,
        "allreduce_ms_per_step": ar_ms,
        "allreduce_bus_gbs": (2.0 * (dist.world - 1) / dist.world * grad_bytes / (ar_ms * 1e-3)
                              / 1e9) if ar_ms > 0 else None,
        "mode": ("replicated features, roots partitioned with batch_offset, then an NCCL "
                 "all-reduce of the dense feature gradient on the compute stream every step "
                 "(the reference's data-parallel usage with torch.distributed)"),
    }


def exchange_leg(w, inp: Inputs, args, dist: Dist, base_ms_per_step: float) -> dict:
    """The replicated step whose backward leaves every rank with the whole
    global batch's feature gradient through exchange regions
    (`sharding.GradientExchange`: every rank publishes its saved ids and
    upstream gradient, every rank adds all ranks' contributions) instead of
    the NCCL all-reduce of the dense gradient.  Checked once against the
    all-reduced gradient (rtol 1e-5 / atol 1e-6), then timed like the main
    step, max over ranks.  Every rank takes the same collective steps."""
    import torch.distributed as tdist

    import fusesampleagg_b200 as fsa
    from fusesampleagg_b200 import sharding

    k1, k2 = w.fanouts
    ex = sharding.GradientExchange(inp.n, w.dim,
                                   sharding.exchange_bytes(w.batch, k1, k2, w.dim),
                                   device=inp.x.device)
    x = inp.x
    x.grad = None
    fsa.fused_sample_agg_2hop(inp.rowptr, inp.col, x, inp.frontiers[0], k1, k2,
                              replay_seed=inp.seeds[0], batch_offset=inp.offset
                              ).backward(inp.grad_out)
    want = x.grad
    x.grad = None
    tdist.all_reduce(want)
    sharding.fused_sample_agg_2hop_exchange(inp.rowptr, inp.col, x, inp.frontiers[0], k1, k2,
                                            replay_seed=inp.seeds[0], batch_offset=inp.offset,
                                            exchange=ex).backward(inp.grad_out)
    torch.cuda.synchronize()
    err = (x.grad - want).abs()
    ok = bool((err <= 1e-6 + 1e-5 * want.abs()).all())
    max_err = float(err.max()) if err.numel() else 0.0
    x.grad = None
    del want, err
    torch.cuda.empty_cache()
    flag = torch.tensor([float(ok)], device="cuda")
    tdist.all_reduce(flag, op=tdist.ReduceOp.MIN)

    class Api:
        @staticmethod
        def fused_sample_agg_2hop(rowptr, col, x, frontier, f1, f2, replay_seed=1234,
                                  batch_offset=0):
            return sharding.fused_sample_agg_2hop_exchange(rowptr, col, x, frontier, f1, f2,
                                                           replay_seed, batch_offset,
                                                           exchange=ex)

    launches0 = fsa.launch_count()
    ms, _ = timed(make_step(Api, w, inp, batch_offset=True), args.steps, args.warmup, dist)
    launches = (fsa.launch_count() - launches0) * args.steps // (args.steps + args.warmup)
    # the same steps with the gradient kept across steps in ex.grad (rows the
    # previous backward touched cleared in the forward, no N x D fill), then
    # one step's ex.grad against the exchanged gradient of the same batch
    ex.persistent = True
    pers_ms, _ = timed(make_step(Api, w, inp, batch_offset=True), args.steps, args.warmup, dist)
    j = (args.warmup + args.steps) % len(inp.frontiers)
    step_j = make_step(Api, w, inp, batch_offset=True)
    step_j(j)
    kept = ex.grad.clone()
    ex.persistent = False
    step_j(j)
    torch.cuda.synchronize()
    pers_ok = bool(torch.isclose(kept, x.grad, rtol=1e-5, atol=1e-6).all())
    x.grad = None
    del kept
    ex.grad = None
    torch.cuda.empty_cache()
    pflag = torch.tensor([float(pers_ok)], device="cuda")
    tdist.all_reduce(pflag, op=tdist.ReduceOp.MIN)
    ex.close()
    units = w.batch * dist.world * args.steps
    per_step = ms / args.steps
    return {
        "value": units / (ms / 1000.0),
        "unit": "roots/s",
        "ms_per_step": per_step,
        "steps": args.steps,
        "warmup": args.warmup,
        "gpu_launches": launches,
        "exchange_ms_per_step": max(per_step - base_ms_per_step, 0.0),
        "grad_matches_allreduce": bool(flag[0].item() == 1.0),
        "grad_check": "every rank's gradient vs the NCCL-all-reduced per-rank gradients, "
                      "rtol 1e-5 / atol 1e-6",
        "grad_max_abs_err_rank0": max_err,
        "persistent_grad": {"value": units / (pers_ms / 1000.0),
                            "ms_per_step": pers_ms / args.steps,
                            "matches_exchanged_gradient": bool(pflag[0].item() == 1.0),
                            "api": "GradientExchange(..., persistent=True): the gradient in "
                                   "exchange.grad, touched rows cleared in the forward"},
        "mode": ("replicated features; the backward publishes this rank's saved ids and "
                 "upstream gradient in an exchange region mapped into every peer (CUDA IPC) and "
                 "adds every rank's contributions into this rank's gradient after a one-float "
                 "NCCL all-reduce: the all-reduced gradient without moving the dense N x D"),
    }


def sharded_leg(w, inp: Inputs, args, dist: Dist) -> dict:
    """The row-sharded mode on the same global batch (2+ GPUs): this rank's
    ids and outputs against the replicated op's for the same slice, bit for
    bit; its gradient shard against the rows it owns of the all-reduced
    replicated gradient (rtol 1e-5 / atol 1e-6); then the same timed step
    through the sharded API.  Every rank takes the same collective steps."""
    import torch.distributed as tdist

    import fusesampleagg_b200 as fsa
    from fusesampleagg_b200 import sharding

    k1, k2 = w.fanouts
    start, stop = sharding.shard_span(inp.n, dist.rank, dist.world)
    feats = sharding.ShardedFeatures(inp.x.detach()[start:stop].clone().requires_grad_(True),
                                     inp.n,
                                     exchange_bytes=sharding.exchange_bytes(w.batch, k1, k2, w.dim))
    exact = True
    checked = min(4, len(inp.frontiers))
    with torch.no_grad():
        for j in range(checked):
            ro, r1, r2 = fsa.fused_sample_agg_2hop_with_samples(
                inp.rowptr, inp.col, inp.x.detach(), inp.frontiers[j], k1, k2,
                replay_seed=inp.seeds[j], batch_offset=inp.offset)
            so, q1, q2 = sharding._forward_2hop_sharded(
                inp.rowptr, inp.col, feats, inp.frontiers[j], k1, k2, inp.seeds[j], True,
                inp.offset, None)
            exact &= (torch.equal(ro.view(torch.int32), so.view(torch.int32))
                      and torch.equal(r1, q1) and torch.equal(r2, q2))
    # gradients: replicated per-rank gradient summed over the ranks vs shards
    inp.x.grad = None
    fsa.fused_sample_agg_2hop(inp.rowptr, inp.col, inp.x, inp.frontiers[0], k1, k2,
                              replay_seed=inp.seeds[0], batch_offset=inp.offset
                              ).backward(inp.grad_out)
    full = inp.x.grad
    inp.x.grad = None
    tdist.all_reduce(full)
    sharding.fused_sample_agg_2hop_sharded(inp.rowptr, inp.col, feats, inp.frontiers[0], k1, k2,
                                           inp.seeds[0], inp.offset).backward(inp.grad_out)
    torch.cuda.synchronize()
    err = (feats.grad - full[start:stop]).abs()
    tol = 1e-6 + 1e-5 * full[start:stop].abs()
    grad_ok = bool((err <= tol).all())
    max_err = float(err.max()) if err.numel() else 0.0
    del full, err, tol
    torch.cuda.empty_cache()
    flags = torch.tensor([float(exact), float(grad_ok)], device="cuda")
    tdist.all_reduce(flags, op=tdist.ReduceOp.MIN)

    class Api:
        @staticmethod
        def fused_sample_agg_2hop(rowptr, col, x, frontier, f1, f2, replay_seed=1234,
                                  batch_offset=0):
            return sharding.fused_sample_agg_2hop_sharded(rowptr, col, feats, frontier, f1, f2,
                                                          replay_seed, batch_offset)

    launches0 = fsa.launch_count()
    ms, _ = timed(make_step(Api, w, inp, batch_offset=True), args.steps, args.warmup, dist)
    launches = (fsa.launch_count() - launches0) * args.steps // (args.steps + args.warmup)
    # the same steps with the backward sent as one remote red.add per
    # contribution (every rank switches together)
    feats.pull = False
    push_ms, _ = timed(make_step(Api, w, inp, batch_offset=True), args.steps, args.warmup, dist)
    feats.pull = True
    # the same steps with the gradient shard kept across steps: each forward
    # clears the rows the previous backward listed instead of zero-filling
    # the shard; then one step's shard against a freshly filled one
    feats.persistent = True
    pers_ms, _ = timed(make_step(Api, w, inp, batch_offset=True), args.steps, args.warmup, dist)
    j = (args.warmup + args.steps) % len(inp.frontiers)
    step_j = make_step(Api, w, inp, batch_offset=True)
    step_j(j)
    kept = feats.grad.clone()
    feats.persistent = False
    step_j(j)
    torch.cuda.synchronize()
    pers_ok = bool(torch.isclose(kept, feats.grad, rtol=1e-5, atol=1e-6).all())
    del kept
    pflag = torch.tensor([float(pers_ok)], device="cuda")
    tdist.all_reduce(pflag, op=tdist.ReduceOp.MIN)
    feats.close()
    del feats
    torch.cuda.empty_cache()
    units = w.batch * dist.world * args.steps
    return {
        "value": units / (ms / 1000.0),
        "unit": "roots/s",
        "ms_per_step": ms / args.steps,
        "steps": args.steps,
        "warmup": args.warmup,
        "bit_exact": bool(flags[0].item() == 1.0),
        "bit_exact_checked": (f"ids (samples1, samples2) and outputs of {checked} root batches "
                              "on every rank against the replicated op on the same slice"),
        "grad_within_tol": bool(flags[1].item() == 1.0),
        "grad_check": ("each rank's gradient shard vs its rows of the NCCL-all-reduced "
                       "replicated gradient, rtol 1e-5 / atol 1e-6"),
        "grad_max_abs_err_rank0": max_err,
        "gpu_launches": launches,
        "push": {"value": units / (push_ms / 1000.0), "ms_per_step": push_ms / args.steps,
                 "backward": "one red.add per remote contribution over NVLink"},
        "persistent_grad": {"value": units / (pers_ms / 1000.0),
                            "ms_per_step": pers_ms / args.steps,
                            "matches_fresh_gradient": bool(pflag[0].item() == 1.0),
                            "clear": ("rows the previous owner-computed backward listed, zeroed "
                                      "inside the sampling kernel instead of the shard's dense "
                                      "fill (ShardedFeatures(persistent=True))")},
        "mode": ("feature rows and their gradient block-sharded over the GPUs: remote rows "
                 "read over NVLink through peer pointers (plain loads, no multicast); backward "
                 "computed by the owners: every rank publishes its saved ids and upstream "
                 "gradient in an exchange region, every rank adds its rows' contributions "
                 "from all regions; one-float NCCL all-reduces order the GPUs"),
    }


def c5_leg(args, dist: Dist, dev) -> dict:
    """The 100M-node scaling configuration (2-hop (15, 10), 1.6B directed
    edges, D = 128, 65,536 roots per GPU): features replicated on one GPU,
    row-sharded over the GPUs (gradient owner-sharded: every rank's
    contributions are added into the owning rank's rows over NVLink) on 2 or
    more.  Device-timed like the main measurement, max over ranks."""
    import fusesampleagg_b200 as api
    from fusesampleagg_b200 import sharding

    w5 = synthetic.WORKLOADS["c5_2hop_100m"]
    t0 = time.time()
    inp = Inputs(w5, dev, dist.rank, dist.world, batches=4)
    setup_s = time.time() - t0
    log(f"[rank {dist.rank}] c5 setup {setup_s:.1f}s graph {inp.stats}")
    same_graph = graph_identical_across_ranks(inp, dist)
    feats = None
    step_api = api
    if dist.world >= 2:
        step_api, feats = sharded_api(inp, w5)
    steps, warmup = min(args.steps, 20), 3
    sampler = ClockSampler(dist.local_rank) if dist.rank == 0 else None
    if sampler:
        sampler.start()
    ms, _ = timed(make_step(step_api, w5, inp, batch_offset=True), steps, warmup, dist, sampler)
    clocks = sampler.stop() if sampler else None
    persistent = None
    if feats is None:
        # the opt-in persistent gradient on the same graph and batches (its
        # buffer replaces the 51 GB dense gradient each step would fill);
        # the last timed step's dense gradient goes first
        inp.x.grad = None
        torch.cuda.empty_cache()
        persistent = persistent_leg(w5, inp, args, dist, check=False, steps=steps, warmup=warmup)
    push = None
    if feats is not None:
        # the backward as one remote red.add per contribution, for comparison
        feats.pull = False
        push_ms, _ = timed(make_step(step_api, w5, inp, batch_offset=True), steps, warmup, dist)
        feats.pull = True
        push = {"value": w5.batch * dist.world * steps / (push_ms / 1000.0),
                "ms_per_step": push_ms / steps,
                "backward": "one red.add per remote contribution over NVLink"}
        # the gradient shards kept across steps, touched rows cleared
        feats.persistent = True
        pers_ms, _ = timed(make_step(step_api, w5, inp, batch_offset=True), steps, warmup, dist)
        feats.persistent = False
        persistent = {"value": w5.batch * dist.world * steps / (pers_ms / 1000.0),
                      "ms_per_step": pers_ms / steps,
                      "clear": "rows the previous backward listed, inside the sampling kernel"}
        feats.close()
    units = w5.batch * dist.world * steps
    out = {
        "value": units / (ms / 1000.0),
        "unit": "roots/s",
        "ms_per_step": ms / steps,
        "steps": steps,
        "warmup": warmup,
        "config": {**w5.describe(), "realized_edges": inp.stats["num_edges"],
                   "realized_max_degree": inp.stats["max_degree"],
                   "roots_per_gpu": w5.batch, "global_batch": w5.batch * dist.world,
                   "graph_identical_across_ranks": same_graph},
        "mode": ("replicated features on one GPU" if feats is None else
                 f"row-sharded features over {dist.world} GPUs (gradient computed by the "
                 "owners from every rank's published ids and upstream gradient)"),
        "push": push,
        "persistent_grad": persistent,
        "setup_s": round(setup_s, 1),
        "clocks": clocks,
    }
    del inp, feats
    torch.cuda.empty_cache()
    return out


def load_reference_op():
    ref_dir = REPO / "oracle" / "_ref" / "fuseop"
    if not (ref_dir / "__init__.py").exists():
        return None
    spec = importlib.util.spec_from_file_location(
        "fuseop", ref_dir / "__init__.py", submodule_search_locations=[str(ref_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["fuseop"] = mod
    spec.loader.exec_module(mod)
    return mod


def run(args) -> None:
    # Both arms run on every rank: the reference is a GPU op, so at N GPUs it
    # gets N GPUs too (each rank times its own slice of roots; the reference
    # API has no batch offset, so its ranks draw their own ids).
    dist = Dist()
    torch.cuda.set_device(dist.local_rank)
    dev = torch.device("cuda", dist.local_rank)
    world = dist.world
    dist.init()
    w = synthetic.WORKLOADS[args.workload]
    if w.hops != 2:
        raise SystemExit("bench.py times the 2-hop workloads")
    if args.impl == "ours":
        import fusesampleagg_b200 as api
    else:
        api = load_reference_op()
        if api is None:
            if dist.rank == 0:
                emit({"impl": "reference",
                      "unavailable": "reference op not built into oracle/_ref "
                                     "(python -m oracle.build --ref)"})
            dist.close()
            return
    batches = args.batches
    inp = Inputs(w, dev, dist.rank, world, batches)
    log(f"[rank {dist.rank}] setup {inp.setup_s:.1f}s graph {inp.stats}")
    same_graph = graph_identical_across_ranks(inp, dist)
    feats = None
    if args.sharded:
        if args.impl != "ours" or world < 2:
            raise SystemExit("--sharded times this package on 2+ GPUs (torchrun)")
        api, feats = sharded_api(inp, w)
    sampler = ClockSampler(dist.local_rank) if dist.rank == 0 else None
    if sampler:
        sampler.start()
    launches0 = api.launch_count() if args.impl == "ours" else None
    step = make_step(api, w, inp, batch_offset=args.impl == "ours")
    if args.allreduce_grad:
        step = with_gradient_allreduce(step, inp)
    ms, _ = timed(step, args.steps, args.warmup, dist, sampler)
    launches = (api.launch_count() - launches0) if args.impl == "ours" else None
    clocks = sampler.stop() if sampler else None
    # Launches counted above include the warm-up steps: report the timed ones.
    if launches is not None:
        launches = launches * args.steps // (args.steps + args.warmup)

    # forward / backward split from a shorter pass with events between them
    # (kept out of the timed region above)
    _, phases = timed(step, min(args.steps, 100), args.warmup, dist, phase_events=True)

    e2e_step, h2d, d2h = make_e2e_step(api, w, inp, batch_offset=args.impl == "ours")
    if args.allreduce_grad:
        e2e_step = with_gradient_allreduce(e2e_step, inp)
    e2e_ms, _ = timed(e2e_step, args.steps, args.warmup, dist)

    units = w.batch * world * args.steps
    value = units / (ms / 1000.0)
    e2e_value = units / (e2e_ms / 1000.0)
    used = sorted({(args.warmup + i) % batches for i in range(args.steps)})
    torch.cuda.empty_cache()  # the steps' cached gradient buffers (51 GB each on C5)
    # (this package's own samples: our arm only -- the reference arm maps none
    # of this repository's libraries)
    bytes_model = (byte_model(w, inp, used[: min(len(used), 16)])
                   if feats is None and args.impl == "ours" else None)
    peak, peak_kind = load_peaks()
    if feats is not None:
        feats.close()

    result = {
        "metric": METRIC,
        "value": value,
        "unit": "roots/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Chung-Lu power-law CSR, N(0,1) features; stand-in for the "
                "reference's OGB/Reddit datasets)",
        "config": {
            **w.describe(),
            "realized_edges": inp.stats["num_edges"],
            "realized_max_degree": inp.stats["max_degree"],
            "size_biased_mean_degree": round(inp.stats["size_biased_mean_degree"], 1),
            "roots_per_gpu": w.batch,
            "global_batch": w.batch * world,
            "root_batches": batches,
            "graph_identical_across_ranks": same_graph,
            "parallelism": (f"roots partitioned over {world} GPU(s), graph replicated, "
                            "feature rows and their gradient block-sharded over the GPUs "
                            "(remote rows read and gradient added over NVLink through peer "
                            "pointers; one-float NCCL all-reduce after forward and backward "
                            "as the cross-GPU ordering)" if feats is not None else
                            f"roots partitioned over {world} GPU(s), graph and features "
                            "replicated, NCCL all-reduce (sum) of the dense N x D feature "
                            "gradient after every backward" if args.allreduce_grad else
                            f"roots partitioned over {world} GPU(s), graph and features "
                            "replicated, no data-path collective"),
            "l2": "inputs larger than L2: x (%.0f MB) gathered at random and the dense "
                  "gradient (%.0f MB) rewritten every step" % (
                      inp.n * w.dim * 4 / 1e6, inp.n * w.dim * 4 / 1e6),
        },
        "phases_ms": phases,
        "e2e": {"value": e2e_value, "unit": "roots/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "copies": "roots + upstream gradient packed in one pinned buffer per root "
                          "batch, one H2D per step issued one step ahead on a copy stream "
                          "(double-buffered), output D2H into pinned memory overlapping the "
                          "next step and read by the host two steps later; the first timed "
                          "step copies its own inputs"},
        "clocks": clocks,
    }
    if args.allreduce_grad:
        result["mode"] = "replicated + gradient all-reduce"
    if feats is not None:
        result["mode"] = "sharded"
        result["gpu_launches"] = launches
    elif args.impl == "ours":
        torch.cuda.empty_cache()
        kt = kernel_times(w, inp, iters=min(args.steps, 30))
        names = {
            "plan": "fsa_2hop_plan_kernel (first hop, second-hop row table)",
            "scan": "fsa_2hop_scan_kernel (chunk prefix over roots)",
            "draw": "fsa_2hop_draw_kernel (second-hop reservoir draws + fused dense-grad "
                    "zero fill)",
            "gather": "fsa_2hop_gather_kernel (winners to ids, two-level mean)",
            "bwd": "fsa_2hop_backward_kernel (replay scatter, red.global.add.v4)",
            "fill": "fsa_fill_zero_kernel (stand-alone zero fill, not in the step)",
        }
        kernels = {}
        launched = ["plan", "draw", "gather", "bwd", "fill"]
        if inp.B >= 2048:  # smaller batches are scanned inside the draw kernel
            launched.insert(1, "scan")
        for name in launched:
            us = kt["fill_alone"] if name == "fill" else kt[name]
            achieved = bytes_model[name] / (us * 1e-6) / 1e9
            kernels[name] = {
                "kernel": names[name],
                "avg_us": us,
                "algorithmic_bytes": int(bytes_model[name]),
                "achieved_gbs": achieved,
                "frac_of_measured_hbm": achieved / peak,
                "frac_of_8tbs": achieved / NOMINAL_HBM_GBS,
            }
        kernels["draw"]["rng_draws_per_launch"] = bytes_model["rng_draws"]
        kernels["draw"]["rng_draws_per_s"] = bytes_model["rng_draws"] / (kt["draw"] * 1e-6)
        kernels["forward_without_fill_us"] = kt["fwd_nofill"]
        kernels["bwd_after_forward_without_fill_us"] = kt["bwd_after_nofill"]
        kernels["bwd_after_forward_writeback_us"] = kt["bwd_after_writeback"]
        rows_bytes = (4.0 * w.dim * bytes_model["valid_leaves"]
                      + 4.0 * inp.B * w.fanouts[0] * w.fanouts[1])
        kernels["zero_rows"] = {
            "kernel": "fsa_zero_rows_kernel (stand-alone clear of one step's saved-id rows, "
                      "as PersistentGradient.zero_() runs it; 20 launches back to back; the "
                      "persistent step clears inside the draw kernel instead)",
            "avg_us": kt["zero_rows"],
            "algorithmic_bytes": int(rows_bytes),
            "achieved_gbs": rows_bytes / (kt["zero_rows"] * 1e-6) / 1e9,
            "frac_of_measured_hbm": rows_bytes / (kt["zero_rows"] * 1e-6) / 1e9 / peak,
        }
        kernels["bwd_sorted_alternative"] = {
            "kernels": "fsa_2hop_sortbwd_{count,scatter,reduce}_kernel + fsa_sortbwd_scan_"
                       "{tiles,totals}_kernel + counts zero fill (sort-by-destination "
                       "backward, not in the step)",
            "avg_us": kt["bwd_sorted"],
            "vs_atomic_bwd": kt["bwd_sorted"] / kt["bwd"],
        }
        dom = max((k for k in launched if k != "fill"), key=lambda k: kt[k])
        traffic = NCU_TRAFFIC.get(args.workload, {}).get(dom)
        result["roofline"] = {
            "kernel": kernels[dom]["kernel"],
            "bound": "hbm",
            "achieved": kernels[dom]["achieved_gbs"],
            "peak": peak,
            "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
            else "fallback 6.65 TB/s",
            "unit": "GB/s",
            "frac": kernels[dom]["achieved_gbs"] / peak,
            "traffic": traffic,
        }
        result["kernels"] = kernels
        # The whole step against the same roofline: every kernel's algorithmic
        # bytes (the 4 N D gradient fill included) over the timed step.
        step_bytes = sum(bytes_model[k] for k in ("plan", "draw", "gather", "bwd"))
        step_gbs = step_bytes / (ms / args.steps * 1e-3) / 1e9
        result["step_roofline"] = {
            "algorithmic_bytes_per_gpu": int(step_bytes),
            "achieved": step_gbs,
            "unit": "GB/s per GPU",
            "peak": peak,
            "frac": step_gbs / peak,
            "note": "fill 4 N D + plan + draws + gather + backward bytes per step and GPU "
                    "over ms_per_step",
        }
        result["unique_leaf_rows_per_batch"] = bytes_model["unique_leaf_rows"]
        result["rng_draws_per_batch"] = bytes_model["rng_draws"]
        result["gpu_launches"] = launches
        if not args.allreduce_grad:
            result["persistent_grad"] = persistent_leg(w, inp, args, dist)
        if dist.rank == 0 and world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(w, inp, budget_s=args.cpu_budget)
    else:
        result["impl"] = "reference"
        result["reference"] = ("the reference's own CUDA op (fuseop/fused_sample_agg.cu + "
                               "fuseop/binding.cpp built for sm_100 from its sources) through "
                               "its public Python API")
        result["cpu_baseline"] = None
        # Only the reference's extension may be mapped in this arm (checked
        # after every step has run).
        result["repo_libraries_mapped"] = check_reference_arm_libraries()
    if args.impl == "ours" and feats is None and not args.allreduce_grad:
        if world >= 2 and not args.no_allreduce_leg:
            result["replicated_allreduce"] = allreduce_leg(w, inp, args, dist, ms / args.steps)
            result["replicated_exchange"] = exchange_leg(w, inp, args, dist, ms / args.steps)
        if world >= 2 and not args.no_sharded_leg:
            result["sharded"] = sharded_leg(w, inp, args, dist)
        if not args.no_c5 and args.workload != "c5_2hop_100m":
            # C2's graph, features and step buffers go before C5 is built
            del step, e2e_step, inp
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            result["c5"] = c5_leg(args, dist, dev)
    dist.close()
    if dist.rank == 0:
        emit(result)


def profile_forward(args) -> None:
    """A fixed, short sequence of C-ABI calls on one GPU for ncu captures:
    `--calls` 2-hop forwards of the workload (different root batches), each
    followed by its backward; `--profile-forward fused` zeroes the gradient
    inside the forward (the step's configuration), `separate` with the
    stand-alone fill kernel, `none` runs forwards only.  `--backward sorted`
    runs the sort-by-destination backward instead of the atomic one.
    `persistent` runs the persistent-gradient step's kernels: the forward
    that zeroes the rows of the previous call's saved ids inside its draw
    kernel (fsa_sample_agg_2hop_forward_zero_rows), then the backward into
    the same buffer.  `onehop`
    runs the 1-hop forward (fanout `--fanout`, with saved ids) and its
    backward into a zeroed gradient on the workload's graph and features."""
    from fusesampleagg_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    w = synthetic.WORKLOADS[args.workload]
    inp = Inputs(w, dev, 0, 1, args.calls)
    if args.profile_forward == "onehop":
        profile_onehop(args, inp, w)
        return
    if args.profile_forward == "pull":
        profile_pull(args, inp, w)
        return
    L = _lib.LIB
    k1, k2 = w.fanouts
    B, D, n = inp.B, w.dim, inp.n
    out = torch.empty((B, D), device=dev)
    s1 = torch.empty((B, k1), dtype=torch.int32, device=dev)
    s2 = torch.empty((B, k1, k2), dtype=torch.int32, device=dev)
    grad = None
    if args.profile_forward != "none":
        # the persistent buffer starts zeroed once; the others are filled per call
        grad = (torch.zeros if args.profile_forward == "persistent" else torch.empty)(
            (n, D), device=dev)
    ws_bytes = L.fsa_sample_agg_2hop_workspace_size(B, k1, k2, 1, 1)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    fused = args.profile_forward == "fused"
    if args.backward == "sorted":
        sws_bytes = L.fsa_sample_agg_2hop_backward_sorted_workspace_size(n, B, k1, k2)
        sws = torch.empty((sws_bytes,), dtype=torch.uint8, device=dev)
    prev_s2 = None
    for j in range(args.calls):
        if args.profile_forward == "persistent":
            # the previous call's rows zeroed inside this call's draw kernel
            _lib.check(L.fsa_sample_agg_2hop_forward_zero_rows(
                inp.rowptr.data_ptr(), inp.col.data_ptr(), n, inp.col.numel(), inp.x.data_ptr(),
                D, inp.frontiers[j].data_ptr(), B, 0, k1, k2, inp.seeds[j], out.data_ptr(),
                s1.data_ptr(), s2.data_ptr(), ws.data_ptr(), ws_bytes, grad.data_ptr(),
                prev_s2.data_ptr() if prev_s2 is not None else None,
                prev_s2.numel() if prev_s2 is not None else 0, stream), "fwd zero rows")
            _lib.check(L.fsa_sample_agg_2hop_backward(
                inp.grad_out.data_ptr(), s1.data_ptr(), s2.data_ptr(), B, D, k1, k2,
                grad.data_ptr(), n, stream), "bwd")
            prev_s2 = s2.clone()
            continue
        if args.profile_forward == "separate":
            _lib.check(L.fsa_fill_zero_f32(grad.data_ptr(), grad.numel(), stream), "fill")
        _lib.check(L.fsa_sample_agg_2hop_forward(
            inp.rowptr.data_ptr(), inp.col.data_ptr(), n, inp.col.numel(), inp.x.data_ptr(), D,
            inp.frontiers[j].data_ptr(), B, 0, k1, k2, inp.seeds[j], out.data_ptr(),
            s1.data_ptr(), s2.data_ptr(), ws.data_ptr(), ws_bytes,
            grad.data_ptr() if fused else None, grad.numel() if fused else 0, stream), "fwd")
        if grad is not None and args.backward == "sorted":
            _lib.check(L.fsa_sample_agg_2hop_backward_sorted(
                inp.grad_out.data_ptr(), s1.data_ptr(), s2.data_ptr(), B, D, k1, k2,
                grad.data_ptr(), n, sws.data_ptr(), sws_bytes, stream), "bwd_sorted")
        elif grad is not None:
            _lib.check(L.fsa_sample_agg_2hop_backward(
                inp.grad_out.data_ptr(), s1.data_ptr(), s2.data_ptr(), B, D, k1, k2,
                grad.data_ptr(), n, stream), "bwd")
        prev_s2 = s2.clone()
    torch.cuda.synchronize()
    emit({"profile_forward": args.profile_forward, "calls": args.calls,
          "backward": args.backward, "workload": args.workload})


def profile_pull(args, inp: Inputs, w) -> None:
    """The owner-computed sharded backward on one GPU: `--shards` exchange
    regions, each holding `--roots` roots of the workload sampled and
    published as one rank would, then `--calls` pull launches for shard 0
    of that many row shards (all regions local: the kernel's own cost
    without NVLink)."""
    from fusesampleagg_b200 import _lib

    import ctypes

    L = _lib.LIB
    dev = inp.x.device
    k1, k2 = w.fanouts
    D, n, W, B = w.dim, inp.n, args.shards, args.roots
    stream = torch.cuda.current_stream().cuda_stream
    need = L.fsa_exchange_bytes(B, k1, k2, D)
    ws_bytes = L.fsa_sample_agg_2hop_workspace_size(B, k1, k2, 1, 1)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=dev)
    out = torch.empty((B, D), device=dev)
    s1 = torch.empty((B, k1), dtype=torch.int32, device=dev)
    s2 = torch.empty((B, k1, k2), dtype=torch.int32, device=dev)
    regions = []
    for r in range(W):
        fr = synthetic.root_batch(n, B, seed=100 + r, device=dev)
        _lib.check(L.fsa_sample_agg_2hop_forward(
            inp.rowptr.data_ptr(), inp.col.data_ptr(), n, inp.col.numel(), inp.x.data_ptr(), D,
            fr.data_ptr(), B, r * B, k1, k2, 7, out.data_ptr(), s1.data_ptr(), s2.data_ptr(),
            ws.data_ptr(), ws_bytes, None, 0, stream), "fwd")
        go = synthetic.features(B, D, seed=200 + r, device=dev)
        reg = torch.empty((need,), dtype=torch.uint8, device=dev)
        _lib.check(L.fsa_sharded_publish_2hop(reg.data_ptr(), need, go.data_ptr(), s1.data_ptr(),
                                              s2.data_ptr(), B, D, k1, k2, stream), "publish")
        regions.append(reg)
    rows = -(-n // W)
    grad = torch.zeros((rows, D), device=dev)
    ptrs = (ctypes.c_void_p * W)(*[r.data_ptr() for r in regions])
    for _ in range(args.calls):
        _lib.check(L.fsa_sample_agg_2hop_backward_sharded_pull(
            ptrs, need, W, 0, grad.data_ptr(), rows, n, D, k1, k2, None, 0, stream), "pull")
    torch.cuda.synchronize()
    emit({"profile_forward": "pull", "calls": args.calls, "shards": W, "roots": B,
          "workload": args.workload})


def profile_onehop(args, inp: Inputs, w) -> None:
    """`--calls` 1-hop forwards (fanout `--fanout`, samples and takes saved)
    of the workload's root batches through the C ABI, each followed by its
    backward into a gradient zeroed once up front."""
    from fusesampleagg_b200 import _lib

    L = _lib.LIB
    B, D, n, k = inp.B, w.dim, inp.n, args.fanout
    dev = inp.x.device
    out = torch.empty((B, D), device=dev)
    samples = torch.empty((B, k), dtype=torch.int32, device=dev)
    takes = torch.empty((B,), dtype=torch.int32, device=dev)
    grad = torch.zeros((n, D), device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    for j in range(args.calls):
        _lib.check(L.fsa_sample_agg_forward(
            inp.rowptr.data_ptr(), inp.col.data_ptr(), n, inp.col.numel(), inp.x.data_ptr(), D,
            inp.frontiers[j].data_ptr(), B, 0, k, inp.seeds[j], out.data_ptr(),
            samples.data_ptr(), takes.data_ptr(), stream), "1-hop fwd")
        _lib.check(L.fsa_sample_agg_backward(
            samples.data_ptr(), takes.data_ptr(), inp.grad_out.data_ptr(), B, D, k,
            grad.data_ptr(), n, stream), "1-hop bwd")
    torch.cuda.synchronize()
    emit({"profile_forward": "onehop", "calls": args.calls, "fanout": k,
          "workload": args.workload})


def main() -> None:
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", default="c2_2hop_powerlaw",
                   choices=[k for k, v in synthetic.WORKLOADS.items() if v.hops == 2])
    p.add_argument("--batches", type=int, default=100)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-budget", type=float, default=12.0)
    p.add_argument("--sharded", action="store_true",
                   help="row-shard the features over the ranks (peer reads over NVLink)")
    p.add_argument("--no-allreduce-leg", action="store_true",
                   help="on 2+ GPUs, skip the replicated step with the NCCL all-reduce of the "
                        "dense feature gradient")
    p.add_argument("--no-sharded-leg", action="store_true",
                   help="on 2+ GPUs, skip the row-sharded check and timing after the main "
                        "measurement")
    p.add_argument("--no-c5", action="store_true",
                   help="skip the 100M-node configuration after the main measurement")
    p.add_argument("--allreduce-grad", action="store_true",
                   help="replicated features: all-reduce the dense feature gradient after "
                        "every backward (NCCL)")
    p.add_argument("--profile-forward",
                   choices=["fused", "separate", "none", "persistent", "onehop", "pull"],
                   help="run a short C-ABI call sequence for ncu instead of the benchmark")
    p.add_argument("--calls", type=int, default=3, help="calls of --profile-forward")
    p.add_argument("--fanout", type=int, default=10, help="fanout of --profile-forward onehop")
    p.add_argument("--shards", type=int, default=8,
                   help="exchange regions (ranks) of --profile-forward pull")
    p.add_argument("--roots", type=int, default=2048,
                   help="roots per exchange region of --profile-forward pull")
    p.add_argument("--backward", choices=["atomic", "sorted"], default="atomic",
                   help="backward variant of --profile-forward")
    args = p.parse_args()
    if args.profile_forward:
        profile_forward(args)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if args.allreduce_grad and (args.sharded or args.impl != "ours" or ws == 1):
        raise SystemExit("--allreduce-grad is the replicated mode's collective: this package "
                         "on 2+ GPUs (torchrun)")
    if args.gpus != ws and ws != 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={ws}")
    if args.gpus > 1 and ws == 1:
        raise SystemExit("launch multi-GPU runs with torchrun (one process per GPU)")
    run(args)


if __name__ == "__main__":
    main()
