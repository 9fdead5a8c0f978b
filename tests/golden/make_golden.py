"""Records golden vectors from the reference's own CUDA op on a B200.

Runs the reference FuseSampleAgg op (its public Python API, built from its
sources into oracle/_ref/fuseop by ``python -m oracle.build --ref``) on every
case of tests/golden/cases.py and writes

* ``reference_b200.npz``: per case the sampled ids (1-hop samples/takes,
  2-hop samples1/samples2), the forward output (small cases) and the feature
  gradient (cases marked grad);
* ``reference_b200.json``: graph/frontier digests, SHA-256 of every forward
  output, the GPU name and the torch/CUDA versions.

Usage (on a machine with a B200 and the built reference):
``python tests/golden/make_golden.py --out <dir>``; the files are then
committed under tests/golden/.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "oracle" / "_ref"))

import fuseop  # noqa: E402  (the reference package built into oracle/_ref)

from tests.golden import cases as C  # noqa: E402


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--out", type=Path, default=REPO / "tests" / "golden")
    args = parser.parse_args()
    assert Path(fuseop.__file__).resolve().is_relative_to(REPO / "oracle" / "_ref"), fuseop.__file__
    dev = torch.device("cuda:0")
    arrays: dict[str, np.ndarray] = {}
    meta = {
        "generator": "tests/golden/make_golden.py",
        "reference_op": "fuseop (reference sources, TORCH_CUDA_ARCH_LIST=10.0)",
        "gpu": torch.cuda.get_device_name(0),
        "torch": torch.__version__,
        "cuda": torch.version.cuda,
        "cases": {},
    }
    graphs = {}
    for case in C.CASES:
        gname = case["graph"]
        if gname not in graphs:
            graphs[gname] = C.GRAPHS[gname]()
        g = graphs[gname]
        frontier = C.frontier_for(gname, g, case["batch"], case["root_seed"])
        x = C.features_for(case, g.num_nodes)
        rowptr, col = g.rowptr.to(dev), g.col.to(dev)
        xd, fd = x.to(dev), frontier.to(dev)
        name = case["name"]
        rec = {"graph_digest": g.digest(), "frontier_sha": sha(frontier)}
        if case["hops"] == 1:
            (k,) = case["fanouts"]
            out, samples, takes = fuseop.fused_sample_agg_with_samples(
                rowptr, col, xd, fd, k, replay_seed=case["seed"])
            arrays[f"{name}/samples"] = samples.cpu().numpy()
            arrays[f"{name}/takes"] = takes.cpu().numpy()
        else:
            k1, k2 = case["fanouts"]
            out, s1, s2 = fuseop.fused_sample_agg_2hop_with_samples(
                rowptr, col, xd, fd, k1, k2, replay_seed=case["seed"])
            arrays[f"{name}/samples1"] = s1.cpu().numpy()
            arrays[f"{name}/samples2"] = s2.cpu().numpy()
        rec["out_sha"] = sha(out)
        if case["store_out"]:
            arrays[f"{name}/out"] = out.cpu().numpy()
        if case["grad"]:
            xg = xd.clone().requires_grad_(True)
            if case["hops"] == 1:
                y = fuseop.fused_sample_agg(rowptr, col, xg, fd, case["fanouts"][0],
                                            replay_seed=case["seed"])
            else:
                y = fuseop.fused_sample_agg_2hop(rowptr, col, xg, fd, *case["fanouts"],
                                                 replay_seed=case["seed"])
            go = C.grad_out_for(case, y.size(0)).to(dev)
            y.backward(go)
            arrays[f"{name}/grad_x"] = xg.grad.cpu().numpy()
        meta["cases"][name] = rec
        print(name, rec["out_sha"][:12], flush=True)
    args.out.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(args.out / "reference_b200.npz", **arrays)
    (args.out / "reference_b200.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
    print("wrote", args.out)


if __name__ == "__main__":
    main()
