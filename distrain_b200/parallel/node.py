"""In-box node runtime: one Distrain node per GPU process.

``InBoxNode`` drives a ``TrainEngine`` through the reference's continuous-training semantics
(node/cli/src/continuous.rs:379-675): train continuously, every ``push_every`` steps extract the
round delta (round-start snapshot - current master), compress it with error feedback and hand it to
the coordinator without stalling the training stream; when a new global checkpoint arrives, push the
partial round (or rebase it onto the checkpoint), swap weights, re-create AdamW, and start a new round.

The data plane is device memory: compressed payloads sit in symmetric (peer-mapped) buffers that the
coordinator's merge kernel reads over NVLink, and new checkpoints are written into every node's
staging buffer by the coordinator's apply+broadcast kernel. The control plane (push metadata,
versions, acknowledgements) goes through the process group's key-value store.
"""
from __future__ import annotations

import torch

from ..config import RunConfig
from ..models.engine import TrainEngine
from ..utils.tracing import nvtx


class BatchFeed:
    """Sequence view of a batch source for ``InBoxNode.train_steps_e2e``: reading element k fetches the
    source's next [batch, seq] int32 batch into pinned host buffer k (of ``depth``, round robin). The loop
    reads element i % depth at step i and waits for step i - 1 before it issues step i + 1, so a buffer is
    refilled only after the copy that read it has completed."""

    def __init__(self, source, batch: int, seq: int, depth: int = 3, accum: int = 1):
        pin = torch.cuda.is_available()
        self.bufs = [torch.empty(accum * batch, seq, dtype=torch.int32) for _ in range(depth)]
        if pin:
            self.bufs = [b.pin_memory() for b in self.bufs]
        self.source = source
        self.batch, self.accum = batch, accum
        self.fetched = 0

    def __len__(self):
        return len(self.bufs)

    def __getitem__(self, k: int) -> torch.Tensor:
        # one step's batch: `accum` consecutive source batches (the micro-batches of the step)
        for a in range(self.accum):
            b = self.source()
            want = (self.batch, self.bufs[k].shape[1])
            if tuple(b.shape) != want:
                raise ValueError(f"batch source gave {tuple(b.shape)}, expected {want}")
            self.bufs[k][a * self.batch:(a + 1) * self.batch].copy_(b)
            self.fetched += 1
        return self.bufs[k]


class InBoxNode:
    def __init__(self, run: RunConfig, rank: int = 0, world: int = 1, device=None, enable_push: bool = True,
                 attn_impl: str = None, tp=None, shard: int = 0, n_shards: int = 1, dp_group=None):
        self.run = run
        self.rank, self.world = rank, world
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if attn_impl is None:
            import os
            attn_impl = os.environ.get("DT_ATTN_IMPL", "dt")
        # tp: a TensorParallel group (this node = one model replica split over the group's GPUs); rank and
        # world then count nodes, and this process runs the protocol for parameter shard `shard` of
        # `n_shards` over `dp_group` (the ranks that hold that shard on every node)
        self.engine = TrainEngine(run.model, run.micro_batch, run.seq_len, optim=run.optim, device=self.device,
                                  seed=run.seed, init_std=run.init_std, attn_impl=attn_impl, tp=tp,
                                  act_ckpt=run.activation_checkpointing, grad_accum=run.grad_accum_steps)
        self.enable_push = enable_push
        self.watchdog = None
        if run.watchdog_step_secs > 0:
            from ..utils.watchdog import StepWatchdog, watchdog_limit
            self.hung = None
            self.watchdog = StepWatchdog(watchdog_limit(run.watchdog_step_secs),
                                         on_timeout=lambda s: setattr(self, "hung", s))
        self.step_count = 0
        self.round_step = 0
        self._graph_ready = False
        # The host may enqueue at most `max_ahead` steps beyond the one the device is running: a merge or
        # swap kernel issued by another thread (on its own, higher-priority stream) is not scheduled ahead
        # of training work already queued on the device, so an unbounded run-ahead would hold it back by
        # the whole queue (measured: ~10 steps, 0.36 s, when 20 steps were enqueued at once).
        self.max_ahead = 2
        self._step_events = []
        self.sync = None
        if enable_push:
            from .inbox import InBoxSync
            self.sync = InBoxSync(self, run, rank, world, self.device, shard=shard, n_shards=n_shards,
                                  dp_group=dp_group)

    def phase_push(self, steps_ahead: int):
        """Place this node's next push ``steps_ahead`` steps from now: the round counter (and the round's
        token count) is set as if the round had begun ``push_every - steps_ahead`` steps ago, and the
        first round's inner-lr warm-up is ended at the full lr. A benchmark uses it so that a push, the
        merge it triggers and the checkpoint swap fall inside its timed steps whatever their number."""
        if self.sync is None:
            return
        pe = self.run.push_every
        self.round_step = max(pe - int(steps_ahead), 0)
        self.sync.round_tokens = self.round_step * self.run.grad_accum_steps * self.run.micro_batch * self.run.seq_len
        if self.sync.first_round:
            self.engine.set_lr(self.run.optim.lr)
            self.sync._lr_set = self.run.optim.lr

    # ── training ──
    def _ensure_graph(self):
        if not self._graph_ready:
            self.engine.capture()
            self._graph_ready = True

    def train_step_device(self, tokens_dev: torch.Tensor):
        """One training step on tokens already resident on the device (no host sync): [A*B, S] int32 with
        A = ``grad_accum_steps`` micro-batches of B = ``micro_batch`` sequences."""
        self._ensure_graph()
        if self.sync is not None and len(self._step_events) >= self.max_ahead:
            self._step_events.pop(0).synchronize()
        with nvtx("step"):
            if self.sync is not None:
                self.sync.before_step()
            self.engine.set_tokens(tokens_dev)
            self.engine.step()
            if self.sync is not None:
                ev = torch.cuda.Event()
                ev.record()
                self._step_events.append(ev)
            if self.watchdog is not None:
                self.watchdog.beat()
            self.step_count += 1
            self.round_step += 1
            if self.sync is not None:
                self.sync.after_step()

    def train_steps_e2e(self, host_batches, steps: int):
        """Public end-to-end loop: pinned-host tokens -> H2D -> step -> D2H loss read, every step.
        The loss of step i is read on the host while step i+1 runs (one step of pipelining)."""
        self._ensure_graph()
        stream = torch.cuda.current_stream()
        pinned_loss = torch.zeros(2, 4, dtype=torch.float32).pin_memory()
        ev = [torch.cuda.Event(), torch.cuda.Event()]
        losses = []
        for i in range(steps):
            with nvtx("step"):
                if self.sync is not None:
                    self.sync.before_step()
                self.engine.ids.copy_(host_batches[i % len(host_batches)], non_blocking=True)
                self.engine.step()
                pinned_loss[i % 2].copy_(self.engine.loss, non_blocking=True)
                ev[i % 2].record(stream)
                self.step_count += 1
                self.round_step += 1
                if self.sync is not None:
                    self.sync.after_step()
            if i > 0:
                ev[(i - 1) % 2].synchronize()
                self._observe(float(pinned_loss[(i - 1) % 2][0]), losses)
        ev[(steps - 1) % 2].synchronize()
        self._observe(float(pinned_loss[(steps - 1) % 2][0]), losses)
        return losses

    def train_stream(self, source, steps: int):
        """``train_steps_e2e`` over a batch source (a callable returning [micro_batch, seq_len] int32 CPU
        tensors, e.g. ``ShardLoader.next_batch``; a step takes ``grad_accum_steps`` of them); returns the
        per-step losses."""
        if getattr(self, "_feed", None) is None or self._feed.source is not source:
            self._feed = BatchFeed(source, self.run.micro_batch, self.run.seq_len, accum=self.run.grad_accum_steps)
        return self.train_steps_e2e(self._feed, steps)

    def _observe(self, loss: float, losses: list):
        losses.append(loss)
        if self.watchdog is not None:
            self.watchdog.beat()
        if self.sync is not None and hasattr(self.sync, "observe_loss"):
            self.sync.per_step_losses = True
            self.sync.observe_loss(loss)

    def close(self):
        if self.watchdog is not None:
            self.watchdog.close()
        if self.sync is not None:
            self.sync.close()
        self.engine.release_graph()
