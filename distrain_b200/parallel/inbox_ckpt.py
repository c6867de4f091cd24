"""Checkpoint persistence and resume for the in-box protocol.

The global checkpoint of the in-box protocol lives in GPU memory (the coordinator's staging slot). Every
``every`` versions the coordinator copies it to the host - in chunks through a pinned bounce buffer on
its merge stream, before the next merge may overwrite the slot - and a writer thread stores it in the
object layout of the reference coordinator (coordinator/src/aggregation.rs:384-424): the fp32 safetensors
model with PyTorch ``[out, in]`` names under ``checkpoints/v{N}/model.safetensors`` plus
``checkpoints/v{N}/metadata.json``, keeping the newest ``keep_versions`` versions
(aggregation.rs:459-501). A tensor-parallel node stores one file per shard,
``checkpoints/v{N}/model-tp{t}of{T}.safetensors`` (local slices of the split tensors;
``gather_checkpoint`` reassembles the reference file). ``resume_flat`` loads the newest stored version
into a node's flat parameter buffer, so a restarted job continues from it.
"""
from __future__ import annotations

import logging
import queue
import re
import threading
from typing import Dict, Optional

import torch

from .. import protocol as P
from ..utils.checkpoint import load_safetensors_bytes, save_safetensors

log = logging.getLogger("distrain_b200.checkpoint")


def shard_checkpoint_path(version: int, shard: int, n_shards: int) -> str:
    if n_shards == 1:
        return P.checkpoint_path(version)
    return f"checkpoints/v{version}/model-tp{shard}of{n_shards}.safetensors"


def stored_versions(store, shard: int = 0, n_shards: int = 1):
    """Versions whose (shard) model file is in the store, ascending."""
    out = []
    for k in store.list_keys("checkpoints/"):
        m = re.match(r"checkpoints/v(\d+)/(.+)$", k)
        if m and k == shard_checkpoint_path(int(m.group(1)), shard, n_shards):
            out.append(int(m.group(1)))
    return sorted(out)


def latest_version(store, n_shards: int = 1) -> Optional[int]:
    """Newest version stored for every shard (None if there is none)."""
    common = None
    for t in range(n_shards):
        vs = set(stored_versions(store, t, n_shards))
        common = vs if common is None else common & vs
    return max(common) if common else None


def resume_flat(store, layout, version: int, shard: int = 0, n_shards: int = 1) -> torch.Tensor:
    """The stored (shard) checkpoint of ``version`` as a flat fp32 CPU buffer in ``layout``'s order."""
    sd = load_safetensors_bytes(store.get(shard_checkpoint_path(version, shard, n_shards)))
    flat = torch.zeros(layout.total, dtype=torch.float32)
    layout.load_state_dict(flat, sd)
    return flat


def gather_checkpoint(store, version: int, n_shards: int) -> Dict[str, torch.Tensor]:
    """The reference-named full state dict of a tensor-parallel checkpoint."""
    from .tensor_parallel import gather_state_dict
    shards = [load_safetensors_bytes(store.get(shard_checkpoint_path(version, t, n_shards))) for t in range(n_shards)]
    return gather_state_dict(shards)


class CheckpointWriter:
    """Host copies of the device checkpoint, written to the object store by a background thread."""

    def __init__(self, store, layout, every: int, keep_versions: int = 10, shard: int = 0, n_shards: int = 1,
                 chunk_elems: int = 16 << 20):
        self.store, self.layout = store, layout
        self.every, self.keep = max(1, int(every)), int(keep_versions)
        self.shard, self.n_shards = shard, n_shards
        self.chunk = int(chunk_elems)
        self._pinned = None
        self.q: "queue.Queue" = queue.Queue(maxsize=1)
        self.written = []
        self.error: Optional[BaseException] = None
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def due(self, version: int) -> bool:
        return version > 0 and version % self.every == 0

    def snapshot(self, theta: torch.Tensor, version: int, stream=None, meta: Optional[dict] = None):
        """Copy ``theta`` (fp32, the layout's flat buffer) to the host now and queue it for writing.
        Blocks while the previous checkpoint is still being written (one in flight)."""
        n = self.layout.total
        host = torch.empty(n, dtype=torch.float32)
        if theta.device.type == "cuda":
            if self._pinned is None:
                self._pinned = torch.empty(min(self.chunk, n), dtype=torch.float32).pin_memory()
            st = stream if stream is not None else torch.cuda.current_stream(theta.device)
            for off in range(0, n, self._pinned.numel()):
                m = min(self._pinned.numel(), n - off)
                with torch.cuda.stream(st):
                    self._pinned[:m].copy_(theta[off:off + m], non_blocking=True)
                st.synchronize()
                host[off:off + m].copy_(self._pinned[:m])
        else:
            host.copy_(theta[:n])
        self.q.put((version, host, dict(meta or {})))

    def _loop(self):
        while True:
            item = self.q.get()
            if item is None:
                return
            version, host, meta = item
            try:
                sd = self.layout.to_state_dict(host)
                self.store.put(shard_checkpoint_path(version, self.shard, self.n_shards), save_safetensors(sd))
                if self.shard == 0:
                    meta.update(version=version, n_shards=self.n_shards)
                    self.store.put_json(P.checkpoint_metadata_path(version), meta)
                self.written.append(version)
                log.info("stored checkpoint v%d (shard %d of %d)", version, self.shard, self.n_shards)
                old = version - self.keep * self.every
                if old > 0:
                    self.store.delete(shard_checkpoint_path(old, self.shard, self.n_shards))
                    if self.shard == 0:
                        self.store.delete(P.checkpoint_metadata_path(old))
            except BaseException as e:  # surfaced by close()
                self.error = e
                log.warning("checkpoint v%d not stored: %r", version, e)
            finally:
                self.q.task_done()

    def close(self):
        self.q.put(None)
        self.thread.join(timeout=600)
        if self.error is not None:
            raise RuntimeError(f"checkpoint writer failed: {self.error!r}") from self.error
