"""Comparison arm: the same trainer with a synchronous NCCL all-reduce of dense fp32 deltas.

The reference has no collective at all: nodes push zstd/JSON sparse deltas over HTTP to a coordinator
(node/cli/src/continuous.rs:532-580 -> coordinator/src/routes.rs:166-404). On one
NVSwitch box the natural baseline for the in-box protocol (compressed deltas pulled by a merge kernel,
checkpoint pushed back with NVLS multimem stores) is plain DiLoCo-style synchronisation with a library
collective: every ``push_every`` steps each rank forms its dense round delta delta = theta_start - theta,
``ncclAllReduce(AVG)`` averages it over all ranks on the training stream, every rank applies
theta = theta_start - outer_lr * mean(delta) (outer lr 1, no momentum: the reference's merge with
uniform weights, no staleness, no compression) and starts a new round, with a fresh AdamW state when
``run.reset_optimizer_on_swap`` is set, as the in-box node does on a checkpoint swap.

It reuses the node's hook points (``before_step`` / ``after_step``) so the benchmark measures exactly
the trainer plus this merge; ``merges`` holds the device time of each all-reduce + apply.
"""
from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist

from .. import ops


class NcclDenseSync:
    def __init__(self, node, run, rank: int, world: int, device, outer_lr: float = 1.0, group=None):
        # world: number of replicas averaged; group: their process group (with tensor parallelism, the
        # ranks holding the same shard of every replica)
        self.node, self.run, self.rank, self.world = node, run, rank, world
        self.group = group
        self.eng = node.engine
        self.outer_lr = float(outer_lr)
        self.snap = self.eng.master.clone()
        self.delta = torch.empty_like(self.snap)
        self.version = 0
        self.seq = 0            # rounds pushed (here: all-reduced), as the in-box node counts its pushes
        self.round_tokens = 0
        self._lr_set = None
        self.first_round = True
        self.coord = None
        self._events: List = []

    def before_step(self):
        # first-round linear warm-up of the inner lr, as the in-box node (reference continuous.rs:588-596)
        o = self.run.optim
        warm = max(int(self.run.push_every * o.warmup_fraction), 2)
        if self.first_round and self.node.round_step < warm:
            self.eng.set_lr(o.lr * self.node.round_step / warm)
        elif self.first_round and self.node.round_step == warm:
            self.eng.set_lr(o.lr)

    def after_step(self):
        if self.node.round_step >= self.run.push_every:
            self._merge()
            self.first_round = False

    def _merge(self):
        eng = self.eng
        train = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(train)
        torch.sub(self.snap, eng.master, out=self.delta)
        if self.world > 1:
            dist.all_reduce(self.delta, op=dist.ReduceOp.AVG, group=self.group)
        eng.master.copy_(self.snap).sub_(self.delta, alpha=self.outer_lr)
        self.snap.copy_(eng.master)
        ops.cast_bf16(eng.master, eng.p16)
        if self.run.reset_optimizer_on_swap:
            eng.m.zero_()
            eng.v.zero_()
            eng.hp[9:11].zero_()
        e1.record(train)
        self._events.append((e0, e1))
        self.version += 1
        self.seq += 1
        self.node.round_step = 0
        self.round_tokens = 0

    @property
    def merges(self):
        """Device ms of each merge (events already completed once the caller has synchronised)."""
        return [{"device_ms": a.elapsed_time(b), "n_contrib": self.world,
                 "pulled_bytes": 0, "broadcast_bytes": 0, "allreduce_bytes": self.delta.numel() * 4,
                 "multicast": False} for a, b in self._events]

    def close(self):
        torch.cuda.synchronize()
