"""In-box asynchronous data plane: node push / coordinator merge / checkpoint swap over device memory.

Every rank is one Distrain node; rank 0 additionally runs the coordinator. Per node:

* ``payload`` - one or two slots of a symmetric (peer-mapped) buffer holding compressed deltas;
* ``staging`` - one fp32 checkpoint slot in a symmetric buffer that the coordinator's broadcast kernel
  writes with NVLS ``multimem.st`` (or per-peer stores); on the coordinator's rank the slot is the global
  checkpoint itself, which the merge updates in place. The coordinator writes version v only after every
  node has swapped to v-1.

Push (node, at a round boundary, reference continuous.rs:532-580): pass A of the compressor on the
training stream (delta + error feedback + re-snapshot, ~0.2 ms), the rest of the compressor on a
side stream into a free payload slot, then a background thread waits for it and posts the push
metadata (the reference ``DeltaPush`` body plus where the payload lives) on the control bus.

Merge (coordinator thread on rank 0): ingest pushes into the ``Accumulator`` (staleness, dedup,
weights), and when the trigger fires run the peer-pull merge kernels on a top-priority stream;
publish the new version. A payload slot is released once its contribution is merged, replaced or
rejected; a node whose next slot is still in use defers the push by a step instead of blocking.

Swap (node, reference continuous.rs:458-502): on a new version push the partial round and copy the
staged checkpoint into the master / bf16 buffers (or, with ``swap_mode="rebase"``, carry the steps since
the last push onto it); re-create AdamW; keep (reference), clear, or fold into the weights the
error-feedback residual.
"""
from __future__ import annotations

import json
import logging
import math
import os
import queue
import threading
import time
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from ..config import RunConfig
from ..protocol import Accumulator, DeltaPush, delta_path
from ..utils.tracing import PhaseTimer, nvtx
from .compression import DeviceCompressor, DevicePayload, adaptive_push_mode
from .inbox_ckpt import CheckpointWriter, latest_version, resume_flat
from .merge import Contribution, DeviceMerger, DistributedMerger
from .partition import merge_stream


log = logging.getLogger("distrain_b200.inbox")


# ─────────────────────────────── control bus ───────────────────────────────
class LocalBus:
    def __init__(self):
        self.d: Dict[str, str] = {}
        self.lock = threading.Lock()

    def set(self, k, v):
        with self.lock:
            self.d[k] = v

    def get(self, k, default=None):
        with self.lock:
            return self.d.get(k, default)


class StoreBus:
    """Key-value control plane over a TCPStore client of the job's rendezvous store."""

    def __init__(self, prefix: str = "dtinbox/"):
        host = os.environ.get("MASTER_ADDR", "127.0.0.1")
        port = int(os.environ.get("MASTER_PORT", "29500"))
        import datetime
        self.store = dist.TCPStore(host, port, is_master=False, timeout=datetime.timedelta(seconds=60))
        self.prefix = prefix
        self.lock = threading.Lock()

    def set(self, k, v):
        with self.lock:
            self.store.set(self.prefix + k, v)

    def get(self, k, default=None):
        with self.lock:
            key = self.prefix + k
            if not self.store.check([key]):
                return default
            return self.store.get(key).decode()

    def wait_get(self, k, timeout: float = 60.0):
        """Blocking read of a key another process is about to set."""
        t0 = time.time()
        while True:
            v = self.get(k)
            if v is not None:
                return v
            if time.time() - t0 > timeout:
                raise TimeoutError(f"control bus key {self.prefix + k} not set within {timeout} s")
            time.sleep(0.0005)


def _symm_alloc(nbytes: int, device, world: int, group=None):
    """Symmetric buffer over `group` (default: the world): (local tensor, peer base pointers by group rank,
    multicast pointer)."""
    if world == 1:
        t = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        return t, [t.data_ptr()], 0, None
    import torch.distributed._symmetric_memory as symm_mem
    t = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
    t.zero_()
    hdl = symm_mem.rendezvous(t, (group or dist.group.WORLD).group_name)
    mc = int(getattr(hdl, "multicast_ptr", 0) or 0)
    if os.environ.get("DT_NO_MULTICAST"):
        mc = 0
    return t, [int(p) for p in hdl.buffer_ptrs], mc, hdl


class InBoxSync:
    """One node's side of the protocol for one parameter shard.

    Without tensor parallelism a node is one GPU and there is one shard. With tensor parallelism
    (``n_shards`` = TP size) every rank of a node runs its own instance for its shard over ``dp_group``
    (the ranks holding that shard on every node): payloads, staging buffers and slot bookkeeping are per
    shard; the coordinator of shard 0 decides merges and publishes a plan that the coordinators of the
    other shards execute with the same coefficients (validation and norm clipping on the full-delta
    norms summed over shards); the ranks of one node swap to a new version at the same step."""

    def __init__(self, node, run: RunConfig, rank: int, world: int, device, shard: int = 0, n_shards: int = 1,
                 dp_group=None):
        self.node, self.run, self.rank, self.world = node, run, rank, world
        self.shard, self.n_shards, self.dp_group = shard, n_shards, dp_group
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        eng = node.engine
        self.eng = eng
        self.layout = eng.layout
        self.n = self.layout.total
        self.node_id = f"node-{rank:02d}"
        self.version = 0
        self.seq = 0
        self.round_tokens = 0
        self.round_loss = []
        self.first_round = True
        self.round_t0 = time.time()
        cfg = run.compression
        self.comp_stream = torch.cuda.Stream(device=self.device)
        # ── symmetric buffers ──
        # bandwidth-adaptive pushes (reference continuous.rs:190-219) may be raw (dense fp32, n values) or
        # loss-based top-k up to 80 %: size the slots for the largest
        kmax = max(cfg.top_k_fraction, 0.80 if run.bandwidth_adaptive else 0.0)
        cap = DeviceCompressor.capacity_for(self.layout, kmax)
        blk = cfg.int8_block if cfg.quantize_int8 else 0
        need = DevicePayload.nbytes(cap, blk)
        if run.bandwidth_adaptive:
            need = max(need, 4 * self.n)
        self.slot_bytes = (need + 4095) // 4096 * 4096
        self.last_loss = float(math.log(run.model.vocab_size))  # previous round's mean loss (adaptive top-k)
        self.loss_ema, self.loss_count = 0.0, 0  # loss-based inner lr (continuous.rs:586-630)
        self.per_step_losses = False             # True once the e2e loop feeds every step's loss
        self._lr_set = None
        # payload slots: with two, a node can push again while the coordinator still holds its previous
        # payload; one is enough when pushes are far apart (and saves ~9 bytes per kept entry)
        self.n_slots = max(1, int(run.payload_slots))
        self.pay_buf, self.pay_ptrs, _, self._pay_h = _symm_alloc(self.n_slots * self.slot_bytes, self.device, world,
                                                                  dp_group)
        self.slots = [DevicePayload(self.pay_buf[i * self.slot_bytes:(i + 1) * self.slot_bytes], cap, blk)
                      for i in range(self.n_slots)]
        # one fp32 checkpoint slot per node (the swap derives the bf16 copy); the coordinator's own slot is
        # its global checkpoint, updated in place by the merge
        self.stage_bytes = (self.n * 4 + 4095) // 4096 * 4096
        self.stage_buf, self.stage_ptrs, self.stage_mc, self._stage_h = _symm_alloc(self.stage_bytes, self.device,
                                                                                   world, dp_group)
        self.compressor = DeviceCompressor(self.layout, self.device, cfg, payload=self.slots[0])
        # checkpoint store: resume from its newest version before anything copies the weights
        self.store = None
        self.resumed_version = 0
        if run.checkpoint_store:  # a directory / file:// path, or an S3 endpoint
            from ..utils.storage import open_store
            self.store = open_store(run.checkpoint_store)
            if run.resume:
                v = latest_version(self.store, n_shards)
                if v:
                    eng.master.copy_(resume_flat(self.store, self.layout, v, shard, n_shards).to(self.device))
                    from .. import ops
                    ops.cast_bf16(eng.master, eng.p16)
                    self.version = self.resumed_version = v
                    log.info("node %s resumed from stored checkpoint v%d", self.node_id, v)
        self.compressor.reset(eng.master)
        # without tensor parallelism every node merges one slice of the checkpoint (DistributedMerger);
        # every node's slot starts as the (identical) initial weights
        self.dm = None
        if n_shards == 1:
            self.ctl, self.ctl_ptrs, _, self._ctl_h = _symm_alloc(DistributedMerger.CTL_BYTES, self.device, world,
                                                                  dp_group)
            self.stage_view().copy_(eng.master)
            self.dm = DistributedMerger(rank, world, self.n, self.device, self.stage_view(), self.stage_ptrs,
                                        self.stage_mc, self.ctl, self.ctl_ptrs,
                                        stream=merge_stream(self.device, run.merge_sms))
        multi = world * n_shards > 1
        self.bus = StoreBus(f"dtinbox/s{shard}/" if n_shards > 1 else "dtinbox/") if multi else LocalBus()
        self.shared = self.bus if n_shards == 1 else StoreBus("dtinbox/shared/")
        if self.resumed_version:
            self.bus.set(f"consumed/{self.rank}", str(self.resumed_version))
        self.inflight = None  # (seq, event, slot)
        self.slot_seq = [-1] * self.n_slots
        self.ef_ready = None
        self.pending_posts: "queue.Queue" = queue.Queue()
        self.stop = threading.Event()
        self.poster = threading.Thread(target=self._post_loop, daemon=True)
        self.poster.start()
        self.latest_version = 0
        self.coord = None
        self.dm_error: Optional[BaseException] = None
        self.dm_thread = None
        if rank == 0:
            self.coord = InBoxCoordinator(self, run, world) if shard == 0 else ShardFollower(self, run, world)
        elif self.dm is not None:
            self.dm_thread = threading.Thread(target=self._dm_loop, daemon=True)
            self.dm_thread.start()
        torch.cuda.synchronize(self.device)
        if world * n_shards > 1:
            dist.barrier()

    # ─────────── helpers ───────────
    def stage_view(self) -> torch.Tensor:
        """This node's fp32 checkpoint slot (on the coordinator's rank: the global checkpoint)."""
        return self.stage_buf[:4 * self.n].view(torch.float32)

    def stage_peer_ptrs(self):
        """(every node's slot by group rank, multicast address of the slots or 0)."""
        return list(self.stage_ptrs), self.stage_mc or 0

    def _slot_free(self, slot: int) -> bool:
        s = self.slot_seq[slot]
        if s < 0:
            return True
        rel = self.bus.get(f"released/{self.rank}/{s}")
        return rel is not None

    # ─────────── step hooks ───────────
    def before_step(self):
        lv = None
        if self.node.step_count % 4 == 0:
            if self.n_shards == 1:
                lv = self.bus.get("version")
            else:
                # the ranks of one node swap at the same step: shard 0 decides, the others read its decision
                key = f"swap/{self.rank}/{self.node.step_count}"
                if self.shard == 0:
                    lv = self.shared.get("version")
                    self.shared.set(key, lv if lv is not None else "-1")
                else:
                    lv = self.shared.wait_get(key)
                    lv = None if lv == "-1" else lv
        if lv is not None and int(lv) > self.version:
            self._swap(int(lv))
        # first-round linear warm-up of the inner lr (reference continuous.rs:588-596), then constant or
        # loss-based
        o = self.run.optim
        warm = max(int(self.run.push_every * o.warmup_fraction), 2)
        if self.first_round and self.node.round_step < warm:
            self.eng.set_lr(o.lr * self.node.round_step / warm)
        elif self.first_round and self.node.round_step == warm:
            self.eng.set_lr(o.lr)
            self._lr_set = o.lr
        elif self.run.loss_based_lr and self.loss_ema > 0.0:
            lr = o.lr * min(max(self.loss_ema / math.log(self.run.model.vocab_size), 0.1), 1.0)
            if self._lr_set is None or abs(lr - self._lr_set) > 1e-3 * lr:
                self.eng.set_lr(lr)
                self._lr_set = lr

    def observe_loss(self, loss: float):
        """One step's (or, without per-step losses, one round's mean) training loss: the EMA behind the
        loss-based inner lr, with the reference's spike rule (continuous.rs:613-630)."""
        if not math.isfinite(loss):
            return
        if self.loss_count > 3 and loss > self.loss_ema * 3.0 and loss > self.loss_ema + 5.0:
            return
        self.loss_count += 1
        self.loss_ema = loss if self.loss_count == 1 else self.loss_ema * 0.9 + loss * 0.1

    def after_step(self):
        self.round_tokens += self.run.grad_accum_steps * self.run.micro_batch * self.run.seq_len
        if self.node.round_step >= self.run.push_every:
            warm = max(int(self.run.push_every * self.run.optim.warmup_fraction), 2)
            if self.first_round and self.node.round_step <= warm:
                return
            if self._push_agreed():
                self.first_round = False

    def _push_agreed(self, partial: bool = False) -> bool:
        """Push now if this shard can (one shard), or as shard 0 decides for every shard of the node, so
        the shards' rounds cover the same steps and carry the same sequence numbers."""
        if self.n_shards == 1:
            return self._push(partial=partial)
        key = f"pushdec/{self.rank}/{self.node.step_count}/{int(partial)}"
        if self.shard == 0:
            mode = self.push_mode()
            ok = self._push(partial=partial, mode=mode)
            self.shared.set(key, json.dumps(list(mode)) if ok else "0")
            return ok
        dec = self.shared.wait_get(key)
        if dec == "0":
            return False
        mode = tuple(json.loads(dec))
        t0 = time.time()
        while not self._push(partial=partial, mode=mode):  # the slot is released for every shard at once
            if time.time() - t0 > 60:
                raise TimeoutError("payload slot of this shard not released")
            time.sleep(0.0005)
        return True

    def push_mode(self):
        """(kind, top-k fraction, int8 block) of the next push (``adaptive_push_mode``); in the box the
        measured bandwidth is the coordinator's payload pull rate over NVLink."""
        bw = float(self.shared.get("bw", "0") or 0.0)
        return adaptive_push_mode(self.run.bandwidth_adaptive, bw, 4 * self.layout.num_params(), self.last_loss,
                                  self.run.compression)

    def _push(self, partial: bool, mode=None) -> bool:
        with nvtx("push"):
            return self._push_impl(partial, mode)

    def _push_impl(self, partial: bool, mode=None) -> bool:
        slot = (self.seq + 1) % self.n_slots
        if not self._slot_free(slot):
            return False  # coordinator still holds that payload; try again next step
        if self.inflight is not None and not self.inflight[1].query():
            return False
        seq = self.seq + 1
        eng = self.eng
        train = torch.cuda.current_stream()
        if self.ef_ready is not None:
            train.wait_event(self.ef_ready)
        kind, kf, qb = mode or self.push_mode()
        self.compressor.begin(eng.master, stream=train)   # pass A on the training stream
        ev_a = torch.cuda.Event()
        ev_a.record(train)
        self.comp_stream.wait_event(ev_a)
        if kind == "raw":
            self.compressor.finish_raw(self.slots[slot].raw(self.n), stream=self.comp_stream)
        else:
            self.compressor.finish(payload=self.slots[slot], stream=self.comp_stream, k_fraction=kf, quant_block=qb)
        ev_f = torch.cuda.Event()
        ev_f.record(self.comp_stream)
        self.ef_ready = ev_f
        ev_l = torch.cuda.Event()
        self.seq = seq
        self.slot_seq[slot] = seq
        steps = self.node.round_step
        tokens = self.round_tokens
        meta = DeltaPush(node_id=self.node_id, seq_num=seq, checkpoint_version=self.version, inner_steps=steps,
                         delta_key=delta_path(self.version, self.node_id, seq), training_loss=0.0,
                         tokens_processed=tokens, training_time_secs=time.time() - self.round_t0)
        # round mean loss: device running sums (loss[2], loss[3]) copied after pass A, then reset
        loss_h = torch.empty(2, dtype=torch.float32).pin_memory()
        self.loss_hold = loss_h
        with torch.cuda.stream(train):
            loss_h.copy_(eng.loss[2:4], non_blocking=True)
            eng.loss[2:4].zero_()
            ev_l.record(train)
        self.comp_stream.wait_event(ev_l)
        ev_post = torch.cuda.Event()
        ev_post.record(self.comp_stream)
        self.inflight = (seq, ev_f, slot)
        self.pending_posts.put((meta, ev_post, slot, loss_h, kind, qb))
        self.node.round_step = 0
        self.round_tokens = 0
        self.round_t0 = time.time()
        return True

    def _post_loop(self):
        torch.cuda.set_device(self.device)
        while not self.stop.is_set():
            try:
                meta, ev, slot, loss_h, kind, qb = self.pending_posts.get(timeout=0.05)
            except queue.Empty:
                continue
            ev.synchronize()
            cnt = float(loss_h[1])
            meta.training_loss = float(loss_h[0]) / cnt if cnt > 0 else 0.0
            if cnt > 0:
                self.last_loss = meta.training_loss
                if not self.per_step_losses:
                    self.observe_loss(meta.training_loss)
            raw = kind == "raw"
            st = self.compressor.read_stats(raw=raw, quantized=qb > 0)
            p = self.slots[slot]
            meta.dense_norm, meta.sparse_norm = st["dense_norm"], st["sparse_norm"]
            meta.compressed_bytes = 4 * st["num_params_kept"] if raw else p.wire_bytes(st["num_params_kept"], qb)
            body = meta.to_dict()
            body["_slot"] = slot
            body["_count"] = st["num_params_kept"]
            body["_rank"] = self.rank
            body["_dense"] = int(raw)
            body["_block"] = qb
            body["_stats"] = st["wire"]  # what the coordinator validates and clips on
            self.bus.set(f"push/{self.rank}/{meta.seq_num}", json.dumps(body))
            self.bus.set(f"pushseq/{self.rank}", str(meta.seq_num))

    def _swap(self, new_version: int):
        t0 = time.perf_counter()
        with nvtx("swap"):
            self._swap_impl(new_version)
        log.info("node %s swap v%d -> v%d in %.1f ms", self.node_id, self.version_before_swap, new_version,
                 (time.perf_counter() - t0) * 1e3)

    def _swap_impl(self, new_version: int):
        self.version_before_swap = self.version
        run = self.run
        rebase = run.swap_mode == "rebase"
        if not rebase and self.node.round_step > 0 and not self.first_round:
            self._push_agreed(partial=True)
        eng = self.eng
        train = torch.cuda.current_stream()
        s32 = self.stage_view()
        fold = run.ef_on_swap == "fold"
        if fold and self.ef_ready is not None:
            train.wait_event(self.ef_ready)  # the in-flight compression has written the residual
        from ..ops._lib import check, stream_ptr, lib, register, c_void, c_ll, c_int
        register("dt_swap_in", [c_void, c_void, c_void, c_void, c_void, c_void, c_ll, c_int, c_void])
        check(lib().dt_swap_in(s32.data_ptr(), None, eng.master.data_ptr(), eng.p16.data_ptr(),
                               self.compressor.snap.data_ptr(), self.compressor.ef.data_ptr() if fold else None,
                               self.n, int(rebase), stream_ptr(train)), "dt_swap_in")
        if run.reset_optimizer_on_swap:  # AdamW re-created (reference continuous.rs:407-414)
            eng.m.zero_()
            eng.v.zero_()
            eng.hp[9:11].zero_()
        if run.ef_on_swap == "reset":
            # cleared after any in-flight compression has read it
            ev = torch.cuda.Event()
            ev.record(train)
            self.comp_stream.wait_event(ev)
            with torch.cuda.stream(self.comp_stream):
                self.compressor.ef.zero_()
            ev2 = torch.cuda.Event()
            ev2.record(self.comp_stream)
            self.ef_ready = ev2
        self.version = new_version
        if not rebase:  # a new round starts at the checkpoint; a rebased round keeps counting
            self.node.round_step = 0
            self.round_tokens = 0
            self.round_t0 = time.time()
        ev_done = torch.cuda.Event()
        ev_done.record(train)
        ev_done.synchronize()
        self.bus.set(f"consumed/{self.rank}", str(new_version))

    def member_contribution(self, m) -> Contribution:
        """A merge member [rank, slot, count, block, weight, dense] as seen from this node (peer pointers)."""
        r, slot, count, blk, weight, dense = m[:6]
        p = self.slots[slot]
        base_local = self.pay_buf.data_ptr()
        peer = self.pay_ptrs[r]
        off = lambda t: t.data_ptr() - base_local + peer
        if dense:
            return Contribution(idx_ptr=0, q_ptr=0, val_ptr=off(p.raw(self.n)), scales_ptr=0, count=self.n, block=0,
                                dense=True, weight=weight, wire_bytes=4 * count)
        return Contribution(idx_ptr=off(p.idx), q_ptr=off(p.q) if blk else 0, val_ptr=off(p.val), win_ptr=off(p.win),
                            scales_ptr=off(p.scales) if blk else 0, count=count, block=blk, dense=False,
                            weight=weight, wire_bytes=p.wire_bytes(count, blk))

    def _dm_loop(self):
        """Nodes other than rank 0: apply this node's slice of every merge attempt rank 0 announces."""
        torch.cuda.set_device(self.device)
        att = 0
        try:
            while not self.stop.is_set():
                raw = self.bus.get(f"dm/{att + 1}")
                if raw is None:
                    time.sleep(0.0005)  # each poll is a store round trip taking the GIL from the training loop
                    continue
                att += 1
                plan = json.loads(raw)
                with nvtx("merge/slice"):
                    self.dm.apply([self.member_contribution(m) for m in plan["members"]], plan["coefs"],
                                  plan["lr"])
                    self.dm.check()
                self.bus.set(f"dmdone/{att}/{self.rank}", "1")
        except BaseException as e:  # surfaced by close()
            self.dm_error = e

    def close(self):
        if self.coord is not None:
            self.coord.close()
        self.stop.set()
        self.poster.join(timeout=5)
        if self.dm_thread is not None:
            self.dm_thread.join(timeout=30)
        torch.cuda.synchronize()
        if self.dm_error is not None:
            raise RuntimeError(f"distributed merge worker failed: {self.dm_error!r}") from self.dm_error


class _Shutdown(Exception):
    pass


class InBoxCoordinator:
    """Coordinator thread on rank 0: ingest pushes, trigger merges, run the device merge, publish versions."""

    def __init__(self, sync: InBoxSync, run: RunConfig, world: int):
        self.sync, self.run, self.world = sync, run, world
        ns = sync.n_shards
        self.bus = sync.bus if isinstance(sync.bus, LocalBus) else StoreBus(sync.bus.prefix)
        # every shard's bus (slot releases, consumed versions) and the cross-shard bus (plans)
        self.shard_buses = [self.bus] if ns == 1 else [StoreBus(f"dtinbox/s{t}/") for t in range(ns)]
        self.shared = self.bus if ns == 1 else StoreBus("dtinbox/shared/")
        self.attempt = 0
        self.acc = Accumulator(staleness_decay=run.staleness_decay, max_staleness=run.max_staleness,
                               min_contributions=0, checkpoint_version=sync.resumed_version)
        self.ckpt = None
        if sync.store is not None and run.checkpoint_every > 0:
            self.ckpt = CheckpointWriter(sync.store, sync.layout, run.checkpoint_every, run.keep_versions, 0,
                                         sync.n_shards)
        from ..coordinator.metrics import Metrics, MetricsServer
        self.metrics = Metrics()
        self.metrics.registered_nodes = world
        self.metrics.checkpoint_version = sync.resumed_version
        self.metrics_server = MetricsServer(self.metrics, port=run.metrics_port) if run.metrics_port >= 0 else None
        for r in range(world):
            self.acc.heartbeat(f"node-{r:02d}")
        self.next_seq = [1] * world
        self.payload_of: Dict[tuple, dict] = {}
        # highest priority: the training graph keeps every SM busy with persistent GEMMs, so merge
        # kernels must be first in line whenever blocks retire or they starve for seconds (the distributed
        # merger has its own such stream)
        self.merger = None
        if sync.dm is None:
            stream = merge_stream(sync.device, run.merge_sms)
            self.merger = DeviceMerger(sync.n, sync.device, sync.eng.master, momentum=0.0, stream=stream,
                                       theta_buffer=sync.stage_view())
        self.version = sync.resumed_version
        self.merges: List[dict] = []
        self.failed: List[str] = []
        self.stop = threading.Event()
        self.error: Optional[BaseException] = None
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def _release(self, rank: int, seq: int):
        for b in self.shard_buses:
            b.set(f"released/{rank}/{seq}", "1")

    def _ingest(self):
        for r in range(self.world):
            while True:
                raw = self.bus.get(f"push/{r}/{self.next_seq[r]}")
                if raw is None:
                    break
                body = json.loads(raw)
                self.next_seq[r] += 1
                push = DeltaPush.from_dict(body)
                prev = [c for c in self.acc.state.contributions if c.node_id == push.node_id]
                ok, reason = self.acc.push(push)
                with self.metrics._lock:
                    self.metrics.delta_pushes_total += 1
                    if ok:
                        self.metrics.delta_pushes_accepted += 1
                    else:
                        self.metrics.delta_pushes_rejected += 1
                    self.metrics.accumulator_contributions = len(self.acc.state.contributions)
                if ok:
                    self.payload_of[(push.node_id, push.seq_num)] = body
                    for c in prev:  # replaced by the newer push from the same node
                        self._release(r, c.seq_num)
                        self.payload_of.pop((c.node_id, c.seq_num), None)
                else:
                    self._release(r, push.seq_num)
                self.acc.heartbeat(push.node_id)

    def _member(self, body: dict, weight: float) -> list:
        p = self.sync.slots[body["_slot"]]
        return [body["_rank"], body["_slot"], body["_count"], body.get("_block", p.block), weight,
                body.get("_dense", 0)]

    def _contribution(self, c) -> Contribution:
        body = self.payload_of[(c.node_id, c.seq_num)]
        out = self.sync.member_contribution(self._member(body, c.weight))
        out.node_id = c.node_id
        return out

    def _wait_consumed(self, version: int, timeout: float = 30.0):
        """Before the merge writes `version` into the single checkpoint slot (in place on this GPU, by
        broadcast on the others), every node of every shard must have swapped to version-1."""
        need = version - 1
        if need < 1:
            return
        t0 = time.time()
        for b in self.shard_buses:
            for r in range(self.world):
                while int(b.get(f"consumed/{r}", "0")) < need:
                    if self.stop.is_set():
                        raise _Shutdown()
                    if time.time() - t0 > timeout:
                        raise TimeoutError(f"node {r} did not consume version {need}")
                    time.sleep(0.001)

    def _merge(self):
        if self.sync.dm is not None:
            return self._merge_distributed()
        snap = self.acc.begin_merge()
        try:
            contribs = [self._contribution(c) for c in snap.contributions]
            new_version = self.version + 1
            self._wait_consumed(new_version)
            p32, mc32 = self.sync.stage_peer_ptrs()
            t0 = time.time()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(self.merger.stream)
            ns = self.sync.n_shards
            self.attempt += 1
            att = self.attempt
            # validation and clipping see the full delta: every shard's push reported the statistics of its
            # payload; sum the squares, take the maxima
            stats = []
            for c in snap.contributions:
                r = int(c.node_id.split("-")[1])
                tot = [0.0, 0.0, 0.0]
                for t in range(ns):
                    if t == 0:
                        body = self.payload_of[(c.node_id, c.seq_num)]
                    else:
                        body = json.loads(self.shard_buses[t].wait_get(f"push/{r}/{c.seq_num}", 120))
                    ss, mx, nf = body["_stats"]
                    tot = [tot[0] + ss, max(tot[1], mx), tot[2] + nf]
                stats.append(tot)
            coefs, info = self.merger.plan(contribs, stats)  # raises when no contribution is valid
            if ns > 1:  # the other shards' coordinators run the same merge on their shards
                self.shared.set(f"plan/{att}", json.dumps({"version": new_version, "coefs": coefs, "members": [
                    [c.node_id, c.seq_num] for c in snap.contributions]}))
            self.merger.accumulate_apply(contribs, coefs, self.run.outer_lr, mc32=mc32, stage32=p32)
            info["pulled_bytes"] = sum(c.wire_bytes for c in contribs)
            ev1.record(self.merger.stream)
            ev1.synchronize()
            for t in range(1, ns):
                self.shared.wait_get(f"merged/{att}/{t}", 120)
            info["device_ms"] = ev0.elapsed_time(ev1)
            info["wall_ms"] = (time.time() - t0) * 1e3
            info["version"] = new_version
            info["n_contrib"] = len(contribs)
            info["broadcast_bytes"] = self.sync.n * 4 * (1 if mc32 else self.world - 1)
            info["multicast"] = bool(mc32)
            self.merges.append(info)
            self._publish_bandwidth(info)
            log.info("merge v%d: %d contributions (%d accepted), %.1f MB pulled, %.2f ms", new_version,
                     len(contribs), info.get("accepted", 0), info.get("pulled_bytes", 0) / 1e6, info["wall_ms"])
            for c in snap.contributions:
                r = int(c.node_id.split("-")[1])
                self._release(r, c.seq_num)
                self.payload_of.pop((c.node_id, c.seq_num), None)
            self.version = new_version
            tokens = sum(c.tokens_processed for c in snap.contributions)
            self.acc.finish_merge(new_version, [c.node_id for c in snap.contributions], tokens)
            self.shared.set("version", str(new_version))
            self._maybe_store(new_version, info)
            self._record(info)
        except _Shutdown:
            self.acc.abort_merge()
            raise
        except Exception as e:
            # like a failed reference aggregation: count it, drop the contributions of this attempt
            # (their payload slots are released) and keep serving
            self.failed.append(repr(e))
            self._record(None, failed=True)
            log.warning("merge failed: %r", e)
            for c in snap.contributions:
                r = int(c.node_id.split("-")[1])
                self._release(r, c.seq_num)
                self.payload_of.pop((c.node_id, c.seq_num), None)
            self.acc.state.contributions = [c for c in self.acc.state.contributions
                                            if (c.node_id, c.seq_num) not in {(x.node_id, x.seq_num)
                                                                             for x in snap.contributions}]
            self.acc.abort_merge()

    def _record(self, info: Optional[dict], failed: bool = False):
        with self.metrics._lock:
            m = self.metrics
            m.aggregations_total += 1
            if failed:
                m.aggregations_failed += 1
                return
            m.checkpoint_version = info["version"]
            m.last_aggregation_secs = info.get("wall_ms", 0.0) / 1e3
            m.merge_device_ms = info.get("device_ms", 0.0)
            m.merge_pulled_bytes = info.get("pulled_bytes", 0)
            m.accumulator_contributions = len(self.acc.state.contributions)
            m.active_nodes = len(self.acc.cs.heartbeats)

    def _maybe_store(self, version: int, info: dict):
        """Persist a due version from this GPU's slot (before the next merge may overwrite it)."""
        if self.ckpt is None or not self.ckpt.due(version):
            return
        stream = self.sync.dm.stream if self.sync.dm is not None else self.merger.stream
        self.ckpt.snapshot(self.sync.stage_view(), version, stream,
                           meta={"contributions_accepted": info.get("accepted"), "source": "in-box merge"})

    def _publish_bandwidth(self, info: dict):
        """Measured payload pull rate of this merge (bytes/s over its wall time), the in-box counterpart of
        the reference node's measured upload bandwidth for bandwidth-adaptive compression."""
        secs = max(info.get("wall_ms", 0.0), 1e-3) / 1e3
        self.shared.set("bw", str(info.get("pulled_bytes", 0) / secs))

    def _wait_key(self, key: str, timeout: float = 120.0):
        t0 = time.time()
        while self.bus.get(key) is None:
            if self.stop.is_set():
                raise _Shutdown()
            if time.time() - t0 > timeout:
                raise TimeoutError(f"control bus key {key} not set within {timeout} s")
            time.sleep(0.0001)

    def _merge_distributed(self):
        """Merge with every node working on its slice (DistributedMerger): announce the members on the bus,
        run this node's share plus the plan, publish the version."""
        snap = self.acc.begin_merge()
        try:
            contribs = [self._contribution(c) for c in snap.contributions]
            members = []
            for c in snap.contributions:
                body = self.payload_of[(c.node_id, c.seq_num)]
                members.append(self._member(body, c.weight))
            new_version = self.version + 1
            self._wait_consumed(new_version)
            dm = self.sync.dm
            timer = PhaseTimer("merge", log)
            with timer.phase("plan"):
                stats = [self.payload_of[(c.node_id, c.seq_num)]["_stats"] for c in snap.contributions]
                coefs, info = DeviceMerger.plan(contribs, stats)  # raises when no contribution is valid
            info["pulled_bytes"] = sum(c.wire_bytes for c in contribs)
            self.attempt += 1
            att = self.attempt
            t0 = time.time()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(dm.stream)
            W = self.world
            lr = self.run.outer_lr
            with timer.phase("announce"):
                if W > 1:
                    self.bus.set(f"dm/{att}", json.dumps({"version": new_version, "members": members,
                                                          "coefs": coefs, "lr": lr}))
            with timer.phase("slice"):
                dm.apply(contribs, coefs, lr)
                dm.check()
            with timer.phase("wait_slices"):
                for r in range(1, W):
                    self._wait_key(f"dmdone/{att}/{r}")
                dm.finish(att)
            info["phases_ms"] = timer.report(version=new_version, contributions=len(contribs))
            ev1.record(dm.stream)
            ev1.synchronize()
            info["device_ms"] = ev0.elapsed_time(ev1)
            info["wall_ms"] = (time.time() - t0) * 1e3
            info["version"] = new_version
            info["n_contrib"] = len(contribs)
            mc = bool(self.sync.stage_mc)
            info["broadcast_bytes"] = self.sync.n * 4 * (1 if mc else max(self.world - 1, 1))
            info["multicast"] = mc
            info["distributed"] = self.world
            self.merges.append(info)
            self._publish_bandwidth(info)
            log.info("merge v%d: %d contributions (%d accepted), %.1f MB pulled, %.2f ms", new_version,
                     len(contribs), info.get("accepted", 0), info.get("pulled_bytes", 0) / 1e6, info["wall_ms"])
            for c in snap.contributions:
                r = int(c.node_id.split("-")[1])
                self._release(r, c.seq_num)
                self.payload_of.pop((c.node_id, c.seq_num), None)
            self.version = new_version
            tokens = sum(c.tokens_processed for c in snap.contributions)
            self.acc.finish_merge(new_version, [c.node_id for c in snap.contributions], tokens)
            self.shared.set("version", str(new_version))
            self._maybe_store(new_version, info)
            self._record(info)
        except _Shutdown:
            self.acc.abort_merge()
            raise
        except Exception as e:
            self.failed.append(repr(e))
            self._record(None, failed=True)
            log.warning("merge failed: %r", e)
            for c in snap.contributions:
                r = int(c.node_id.split("-")[1])
                self._release(r, c.seq_num)
                self.payload_of.pop((c.node_id, c.seq_num), None)
            self.acc.state.contributions = [c for c in self.acc.state.contributions
                                            if (c.node_id, c.seq_num) not in {(x.node_id, x.seq_num)
                                                                             for x in snap.contributions}]
            self.acc.abort_merge()

    def _loop(self):
        torch.cuda.set_device(self.sync.device)
        try:
            while not self.stop.is_set():
                self._ingest()
                if self.acc.ready():
                    self._merge()
                else:
                    time.sleep(0.0005)
        except _Shutdown:
            pass
        except BaseException as e:  # surfaced by close()
            self.error = e

    def close(self):
        self.stop.set()
        self.thread.join(timeout=30)
        if self.ckpt is not None:
            self.ckpt.close()
        if self.metrics_server is not None:
            self.metrics_server.stop()
        if self.error is not None:
            raise RuntimeError(f"coordinator thread failed: {self.error!r}") from self.error


class ShardFollower:
    """Coordinator thread for shard t > 0 (on node 0's rank of that shard): executes the merge plans of the
    shard-0 coordinator (members and coefficients, planned on the full-delta statistics of all shards) on
    this shard's payloads - accumulate + apply + broadcast into this shard's staging buffers - and reports
    completion. Slot releases and version publication are the shard-0 coordinator's."""

    def __init__(self, sync: InBoxSync, run: RunConfig, world: int):
        self.sync, self.run, self.world = sync, run, world
        self.bus = StoreBus(sync.bus.prefix)
        self.shared = StoreBus("dtinbox/shared/")
        stream = merge_stream(sync.device, run.merge_sms)
        self.merger = DeviceMerger(sync.n, sync.device, sync.eng.master, momentum=0.0, stream=stream,
                                   theta_buffer=sync.stage_view())
        self.ckpt = None
        if sync.store is not None and run.checkpoint_every > 0:
            self.ckpt = CheckpointWriter(sync.store, sync.layout, run.checkpoint_every, run.keep_versions, sync.shard,
                                         sync.n_shards)
        self.attempt = 0
        self.merges: List[dict] = []
        self.failed: List[str] = []
        self.stop = threading.Event()
        self.error: Optional[BaseException] = None
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def _contribution(self, node_id: str, seq: int) -> Contribution:
        r = int(node_id.split("-")[1])
        body = json.loads(self.bus.wait_get(f"push/{r}/{seq}", 120))
        p = self.sync.slots[body["_slot"]]
        out = self.sync.member_contribution([r, body["_slot"], body["_count"], body.get("_block", p.block), 1.0,
                                             body.get("_dense", 0)])
        out.node_id = node_id
        return out

    def _one(self, att: int, plan: dict):
        v = plan["version"]
        contribs = [self._contribution(nid, seq) for nid, seq in plan["members"]]
        p32, mc32 = self.sync.stage_peer_ptrs()
        self.merger.accumulate_apply(contribs, plan["coefs"], self.run.outer_lr, mc32=mc32, stage32=p32)
        self.merger.stream.synchronize()
        self.merges.append({"version": v, "n_contrib": len(contribs)})
        if self.ckpt is not None and self.ckpt.due(v):  # this shard's file, before the next merge writes
            self.ckpt.snapshot(self.sync.stage_view(), v, self.merger.stream)
        self.shared.set(f"merged/{att}/{self.sync.shard}", "1")

    def _loop(self):
        torch.cuda.set_device(self.sync.device)
        try:
            while not self.stop.is_set():
                raw = self.shared.get(f"plan/{self.attempt + 1}")
                if raw is None:
                    time.sleep(0.0005)
                    continue
                self.attempt += 1
                self._one(self.attempt, json.loads(raw))
        except BaseException as e:  # surfaced by close()
            self.error = e

    def close(self):
        self.stop.set()
        self.thread.join(timeout=30)
        if self.ckpt is not None:
            self.ckpt.close()
        if self.error is not None:
            raise RuntimeError(f"shard coordinator thread failed: {self.error!r}") from self.error
