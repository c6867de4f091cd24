"""Loss gap of the asynchronous protocol to single-GPU training at matched tokens.

    # N nodes (one per GPU), `steps` steps each, the full in-box protocol (push every P, merge, swap):
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \\
        -m distrain_b200.bench_loss --config tiny --steps S --data markov
    # the single-GPU baseline at matched tokens (N * S steps, no pushes):
    python -m distrain_b200.bench_loss --config tiny --steps N*S --data markov

Data: ``uniform`` (the benchmark's uniform-random token ids: every model's loss is ln(vocab)) or ``markov``:
a fixed random first-order Markov chain over the vocabulary (each token has 4 successors with fixed
probabilities, entropy ~1.3 nats), which a model can learn, so the gap measures what the protocol costs.
Every rank draws its own sequences (per-rank seed) from the same chain. At the end every rank evaluates
the model it holds on the same held-out batches (forward loss, no update); rank 0 prints one JSON line with
the final held-out loss (max and mean over ranks), the training loss of the last steps and the number of
merges. The loss gap is the multi-node held-out loss minus the single-GPU one at the same tokens.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist


class MarkovTokens:
    """First-order Markov chain over [0, vocab): token t is followed by succ[t, j] with probability p[j]."""

    def __init__(self, vocab: int, batch: int, seq_len: int, seed: int, chain_seed: int = 12345, branching: int = 4):
        cg = np.random.default_rng(chain_seed)
        self.succ = cg.integers(0, vocab, size=(vocab, branching), dtype=np.int64)
        w = np.array([0.55, 0.25, 0.12, 0.08][:branching], dtype=np.float64)
        self.cdf = np.cumsum(w / w.sum())
        self.rng = np.random.default_rng(seed)
        self.vocab, self.batch, self.seq_len = vocab, batch, seq_len

    def entropy(self) -> float:
        p = np.diff(np.concatenate([[0.0], self.cdf]))
        return float(-(p * np.log(p)).sum())

    def next_batch(self) -> torch.Tensor:
        B, S = self.batch, self.seq_len
        out = np.empty((B, S), dtype=np.int64)
        out[:, 0] = self.rng.integers(0, self.vocab, size=B)
        u = self.rng.random((B, S - 1))
        j = np.searchsorted(self.cdf, u)
        for t in range(1, S):
            out[:, t] = self.succ[out[:, t - 1], j[:, t - 1]]
        return torch.from_numpy(out.astype(np.int32))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="tiny")
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--data", default="markov", choices=["markov", "uniform"])
    ap.add_argument("--push-every", type=int, default=None)
    ap.add_argument("--eval-batches", type=int, default=4)
    ap.add_argument("--swap-mode", default=None, choices=["push_partial", "rebase"])
    ap.add_argument("--ef-on-swap", default=None, choices=["keep", "reset", "fold"])
    ap.add_argument("--reset-optimizer", default=None, choices=["yes", "no"],
                    help="re-create the AdamW state at checkpoint swaps (the reference node does)")
    ap.add_argument("--topk", type=float, default=None, help="top-k fraction of the delta compression")
    ap.add_argument("--sync", default="inbox", choices=["inbox", "nccl"],
                    help="inbox: the compressed asynchronous protocol; nccl: dense synchronous delta averaging")
    a = ap.parse_args()
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from distrain_b200.config import bench_config
    from distrain_b200.parallel.node import InBoxNode
    from distrain_b200.utils.data import SyntheticTokens

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=300))
    run = bench_config(a.config)
    if a.push_every:
        run.push_every = a.push_every
    if a.swap_mode:
        run.swap_mode = a.swap_mode
    if a.ef_on_swap:
        run.ef_on_swap = a.ef_on_swap
    if a.reset_optimizer:
        run.reset_optimizer_on_swap = a.reset_optimizer == "yes"
    if a.topk:
        run.compression.top_k_fraction = a.topk
    node = InBoxNode(run, rank=rank, world=world, device=dev, enable_push=world > 1 and a.sync == "inbox")
    if world > 1 and a.sync == "nccl":
        from distrain_b200.parallel.nccl_baseline import NcclDenseSync
        node.sync = NcclDenseSync(node, run, rank, world, dev)
    B, S, V = run.micro_batch, run.seq_len, run.model.vocab_size
    mk = (lambda seed: MarkovTokens(V, B, S, seed)) if a.data == "markov" else \
        (lambda seed: SyntheticTokens(V, B, S, seed))
    gen = mk(1000 + rank)
    ring = [gen.next_batch().pin_memory() for _ in range(2)]
    losses = []
    for i in range(a.steps):
        losses.extend(node.train_steps_e2e([ring[i % 2]], 1))
        ring[i % 2] = gen.next_batch().pin_memory()  # next batch prepared while the GPU runs
    torch.cuda.synchronize()
    merges = 0
    if node.sync is not None:
        if a.sync == "nccl":
            merges = len(node.sync.merges)
        elif node.sync.coord is not None:
            merges = len(node.sync.coord.merges)
    version = node.sync.version if node.sync is not None else 0
    if node.sync is not None:
        node.sync.close()
        node.sync = None
    node.engine.release_graph()
    # held-out evaluation of the model this rank holds (same batches on every rank)
    ev = mk(999_999)
    eng = node.engine
    saved = (eng.master.clone(), eng.m.clone(), eng.v.clone(), eng.hp.clone())
    tot = 0.0
    for _ in range(a.eval_batches):
        eng.set_tokens(ev.next_batch().to(dev))
        eng.forward_backward()
        tot += float(eng.loss[0])
    eng.master.copy_(saved[0]); eng.m.copy_(saved[1]); eng.v.copy_(saved[2]); eng.hp.copy_(saved[3])
    held = torch.tensor([tot / a.eval_batches, tot / a.eval_batches], device=dev, dtype=torch.float64)
    if world > 1:
        mx = held.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(held, op=dist.ReduceOp.SUM)
        held = torch.stack([mx[0], held[1] / world])
    if rank == 0:
        tail = losses[-20:]
        out = {"bench": "loss_gap", "config": a.config, "data": a.data, "n_nodes": world, "steps_per_node": a.steps,
               "tokens_total": a.steps * B * (S - 1) * world, "heldout_loss_max": round(float(held[0]), 4),
               "heldout_loss_mean": round(float(held[1]), 4), "train_loss_last20": round(sum(tail) / len(tail), 4),
               "merges": merges, "global_version": version, "push_every": run.push_every if world > 1 else None}
        if world > 1:
            out.update(sync=a.sync, reset_optimizer_on_swap=run.reset_optimizer_on_swap)
            if a.sync == "inbox":
                out.update(swap_mode=run.swap_mode, ef_on_swap=run.ef_on_swap,
                           top_k=run.compression.top_k_fraction)
        if a.data == "markov":
            out["entropy_floor"] = round(gen.entropy(), 4)
        else:
            out["entropy_floor"] = round(float(np.log(V)), 4)
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
