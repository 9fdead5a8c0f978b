"""Forward-only 2-hop microbenchmark with the same workload, command line and
JSON fields as the reference's `bench/microbench_2hop.py:11-68`, so the two
numbers can be read side by side.

Workload: a regular CSR graph (every row `--degree` neighbours drawn
uniformly with replacement, `torch.manual_seed(--seed)` on the CPU), N(0,1)
features, `--batch-size` roots drawn with replacement, fanouts (15, 10), one
forward per step with replay seed `seed + step`, under `torch.no_grad()`.
The graph, features and roots come from the same torch generator calls in
the same order as the reference script, so both implementations sample the
same neighbours.

    python -m fusesampleagg_b200.microbench_2hop [--impl ours|reference] ...

prints ``{"mean_step_ms": ..., "sampled_edges_per_second": ..., "steps": ...}``
(plus ``"impl"``), where sampled edges = batch x fanout1 x fanout2 per step.
``--impl reference`` runs the reference op built from its sources into
``oracle/_ref`` when that build exists.  ``--kernel-times`` (this package
only) adds the per-kernel CUDA-event times of the forward and the gather
kernel's algorithmic bandwidth: second-hop winner ids and their col entries
(4 B each), the valid leaf rows (4·D B each) and the output (4·D B per
root), against the measured HBM copy bandwidth in MEASURED_PEAKS.json when
the repository holds one.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parents[1]


def regular_graph(num_nodes: int, degree: int, device: str = "cuda"):
    """rowptr = 0, d, 2d, ...; col = `num_nodes * degree` uniform ids, in
    generation order (rows are not sorted, as in the reference script)."""
    rowptr = torch.arange(0, (num_nodes + 1) * degree, degree, dtype=torch.int32)
    col = torch.randint(0, num_nodes, (num_nodes * degree,), dtype=torch.int32)
    return rowptr.to(device), col.to(device)


def make_inputs(nodes: int, features: int, degree: int, batch: int, seed: int,
                device: str = "cuda"):
    """Graph, features and roots from the seeded default generator, in the
    reference script's order: CSR (CPU), features (device), roots (device)."""
    torch.manual_seed(seed)
    rowptr, col = regular_graph(nodes, degree, device)
    x = torch.randn(nodes, features, device=device)
    roots = torch.randint(0, nodes, (batch,), dtype=torch.int32, device=device)
    return rowptr, col, x, roots


def load_op(impl: str):
    if impl == "ours":
        import fusesampleagg_b200 as ours

        return ours.fused_sample_agg_2hop
    ref_dir = REPO / "oracle" / "_ref" / "fuseop"
    if not (ref_dir / "__init__.py").exists():
        return None
    spec = importlib.util.spec_from_file_location(
        "fuseop", ref_dir / "__init__.py", submodule_search_locations=[str(ref_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["fuseop"] = mod
    spec.loader.exec_module(mod)
    return mod.fused_sample_agg_2hop


@torch.no_grad()
def run(args) -> dict:
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required")
    op = load_op(args.impl)
    if op is None:
        return {"impl": args.impl, "unavailable": "reference op not built into oracle/_ref"}
    rowptr, col, x, roots = make_inputs(args.nodes, args.features, args.degree,
                                        args.batch_size, args.seed)
    f1, f2 = args.fanout
    for step in range(args.warmup):
        op(rowptr, col, x, roots, f1, f2, args.seed + step)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for step in range(args.steps):
        op(rowptr, col, x, roots, f1, f2, args.seed + args.warmup + step)
    end.record()
    end.synchronize()
    ms = start.elapsed_time(end)
    edges = args.batch_size * f1 * f2 * args.steps
    res = {"impl": args.impl, "mean_step_ms": ms / args.steps,
           "sampled_edges_per_second": edges / (ms / 1000.0), "steps": args.steps}
    if getattr(args, "kernel_times", False) and args.impl == "ours":
        res["kernels"] = kernel_times(op, rowptr, col, x, roots, f1, f2, args)
    return res


def measured_hbm_gbs() -> tuple[float, str]:
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
        return float(peaks["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


def kernel_times(op, rowptr, col, x, roots, f1, f2, args) -> dict:
    """Per-kernel times of `args.steps` more forwards (the library's phase
    events) and the gather kernel's algorithmic GB/s."""
    from . import _lib

    _lib.phase_timing(True)
    try:
        for step in range(args.steps):
            op(rowptr, col, x, roots, f1, f2, args.seed + step)
        torch.cuda.synchronize()
        ms, calls = _lib.phase_times()
    finally:
        _lib.phase_timing(False)
    us = {k: 1000.0 * v / calls for k, v in ms.items()}
    # valid second-hop leaves of one call: every slot of a row whose take is
    # positive holds a valid id (the ids come from the op itself)
    from . import fused_sample_agg_2hop_with_samples

    _, _, s2 = fused_sample_agg_2hop_with_samples(rowptr, col, x, roots, f1, f2, args.seed)
    valid = int((s2 >= 0).sum())
    B, D = roots.numel(), x.size(1)
    gather_bytes = 4 * B * f1 * f2 + 4 * valid + 4 * D * valid + 4 * D * B
    gbs = gather_bytes / (us["gather"] * 1e-6) / 1e9
    peak, kind = measured_hbm_gbs()
    return {"plan_us": us["plan"], "scan_us": us["scan"], "draw_us": us["draw"],
            "gather_us": us["gather"],
            "valid_leaves": valid, "gather_algorithmic_bytes": gather_bytes,
            "gather_gbs": gbs, "peak_gbs": peak, "peak_kind": kind,
            "gather_frac_of_peak": gbs / peak}


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--nodes", type=int, default=1_000_000)
    p.add_argument("--features", type=int, default=128)
    p.add_argument("--degree", type=int, default=20)
    p.add_argument("--batch-size", type=int, default=4096)
    p.add_argument("--fanout", nargs=2, type=int, default=[15, 10])
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--kernel-times", action="store_true",
                   help="add per-kernel times and the gather kernel's bandwidth (ours)")
    print(json.dumps(run(p.parse_args(argv)), sort_keys=True))


if __name__ == "__main__":
    main()
