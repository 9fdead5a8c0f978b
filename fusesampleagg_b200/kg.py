"""Knowledge-graph encoder training step around the fused 2-hop operator.

The pattern of the reference's link-prediction benchmark
(`train/kg_completion_bench.py:96-147` model, `:300-336` step): the batch's
head and tail entities are deduplicated (`torch.unique`), each unique
entity's 2-hop neighbourhood mean comes from the fused operator over the
trainable entity table, a two-layer MLP combines it with the entity's own
embedding, DistMult scores the (head, relation, tail) triples against
uniformly drawn negative tails, binary cross-entropy is the loss and AdamW
steps every parameter — the entity table included, through the operator's
backward.

Data are synthetic stand-ins for the reference's OGB knowledge graphs
(absent here): the adjacency is a seeded power-law graph with the C4 shapes
(94k entities / 10.2M adjacency entries / D=200, or 2.5M / 32M / D=100),
training triples are its edges with seeded relation ids.

    python -m fusesampleagg_b200.kg [--impl ours|reference] [--workload c4a_kg_2hop]

prints one JSON line with the training throughput in triples/s.
"""

from __future__ import annotations

import argparse
import json
import time

import torch
import torch.nn.functional as F
from torch import nn

from . import synthetic


class KGEncoder(nn.Module):
    """Entity and relation embeddings plus the neighbourhood-mean MLP."""

    def __init__(self, num_entities: int, num_relations: int, dim: int, init_std: float = 0.1):
        super().__init__()
        self.entities = nn.Embedding(num_entities, dim)
        self.relations = nn.Embedding(num_relations, dim)
        nn.init.normal_(self.entities.weight, std=init_std)
        nn.init.normal_(self.relations.weight, std=init_std)
        self.projection = nn.Sequential(nn.Linear(2 * dim, dim), nn.ReLU(), nn.Linear(dim, dim))

    def encode(self, entity_ids, rowptr, col, fanout1, fanout2, seed, op):
        unique, inverse = torch.unique(entity_ids.long(), return_inverse=True)
        neighbour_mean = op(rowptr, col, self.entities.weight, unique.to(torch.int32),
                            fanout1, fanout2, replay_seed=seed)
        encoded = self.projection(torch.cat([self.entities(unique), neighbour_mean], dim=-1))
        return encoded[inverse]

    @staticmethod
    def score(head, relation, tail):
        return (head * relation * tail).sum(dim=-1)


class KGData:
    """Seeded synthetic triples over a workload's adjacency."""

    def __init__(self, workload: str, num_relations: int = 64, seed: int = 0, device="cuda"):
        w = synthetic.WORKLOADS[workload]
        self.workload = w
        g = w.graph(seed, device)
        self.rowptr, self.col = g.rowptr, g.col
        self.num_entities = g.num_nodes
        self.num_relations = num_relations
        deg = (g.rowptr[1:] - g.rowptr[:-1]).long()
        # every adjacency entry (row -> col) is a training triple
        self.heads = torch.repeat_interleave(torch.arange(g.num_nodes, device=device), deg)
        self.tails = g.col.long()
        gen = torch.Generator(device=device).manual_seed(seed + 17)
        self.relations = torch.randint(0, num_relations, (self.heads.numel(),), device=device,
                                       generator=gen)
        self.gen = torch.Generator(device=device).manual_seed(seed + 29)

    def batch(self, size: int, negatives: int):
        idx = torch.randint(0, self.heads.numel(), (size,), device=self.heads.device,
                            generator=self.gen)
        neg = torch.randint(0, self.num_entities, (size, negatives), device=self.heads.device,
                            generator=self.gen)
        return self.heads[idx], self.relations[idx], self.tails[idx], neg


def make_train_step(model: KGEncoder, data: KGData, op, fanouts, batch: int, negatives: int,
                    lr: float = 3e-4):
    """One step: encode heads and tails, DistMult against the true and
    negative tails, BCE, AdamW.  Returns (step(i) -> loss tensor, optimizer)."""
    opt = torch.optim.AdamW(model.parameters(), lr=lr, weight_decay=1e-4)
    f1, f2 = fanouts

    def step(i: int) -> torch.Tensor:
        head, rel, tail, neg = data.batch(batch, negatives)
        z = model.encode(torch.cat([head, tail]), data.rowptr, data.col, f1, f2,
                         1_000_003 + i, op)
        hz, tz = z[:batch], z[batch:]
        rz = model.relations(rel)
        pos = model.score(hz, rz, tz)
        negs = (hz[:, None, :] * rz[:, None, :] * model.entities(neg)).sum(dim=-1)
        loss = F.binary_cross_entropy_with_logits(pos, torch.ones_like(pos))
        loss = loss + F.binary_cross_entropy_with_logits(negs, torch.zeros_like(negs))
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        return loss.detach()

    return step, opt


def load_op(impl: str):
    if impl == "ours":
        import fusesampleagg_b200 as fsa

        return fsa.fused_sample_agg_2hop
    from .microbench_2hop import load_op as mb_load

    return mb_load("reference")


def run(args) -> dict:
    op = load_op(args.impl)
    if op is None:
        return {"impl": args.impl, "unavailable": "reference op not built into oracle/_ref"}
    torch.manual_seed(args.seed)
    data = KGData(args.workload, seed=args.seed)
    w = data.workload
    model = KGEncoder(data.num_entities, data.num_relations, w.dim).cuda()
    step, _ = make_train_step(model, data, op, w.fanouts, args.batch_size, args.negatives)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    start.record()
    loss = None
    for i in range(args.steps):
        loss = step(args.warmup + i)
    end.record()
    end.synchronize()
    ms = start.elapsed_time(end)
    return {"metric": "kg train triples/s", "impl": args.impl,
            "value": args.batch_size * args.steps / (ms / 1000.0), "unit": "triples/s",
            "ms_per_step": ms / args.steps, "steps": args.steps, "warmup": args.warmup,
            "final_loss": float(loss), "wall_s": time.time() - t0,
            "config": {"workload": args.workload, "entities": data.num_entities,
                       "adjacency_entries": int(data.col.numel()), "dim": w.dim,
                       "fanouts": list(w.fanouts), "batch_size": args.batch_size,
                       "negatives": args.negatives, "relations": data.num_relations,
                       "optimizer": "AdamW lr 3e-4 wd 1e-4", "data": "synthetic"}}


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", default="c4a_kg_2hop",
                   choices=["c4a_kg_2hop", "c4b_kg_2hop"])
    p.add_argument("--batch-size", type=int, default=512)
    p.add_argument("--negatives", type=int, default=64)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--seed", type=int, default=0)
    print(json.dumps(run(p.parse_args(argv))))


if __name__ == "__main__":
    main()
