"""Training data: uint16 token shards + manifest (reference node/cli/src/data.rs, scripts/prepare_data.py).

* ``tokenize_to_shards`` - text documents (local .txt / .jsonl / .parquet files) through a
  ``tokenizers`` JSON tokenizer into the same shard format (the reference's tokenize-and-shard step).
* ``write_shard`` / ``write_manifest`` / ``prepare_random_shards`` - the data-prep format: flat LE
  uint16 files ``shard_XXXX.bin`` and ``manifest.json`` = {num_shards, vocab_size, shards[{filename,
  num_tokens, size_bytes}], total_tokens}.
* ``ShardLoader`` - the native loader (mmap, sequential wrap-around batches, seek_by_seed, bounded
  resident window, background prefetch into pinned buffers).
* ``StreamingLoader`` - fetches assigned shards from an object store into a local cache, then reads them
  through ``ShardLoader`` (reference StreamingDataLoader / download_shard_cached).
* ``SyntheticTokens`` - seeded uniform-random token batches (the benchmark data).
"""
from __future__ import annotations

import ctypes
import json
import logging
import os
from typing import List, Optional

import numpy as np
import torch

from .native import rt, register, NativeError
from .. import protocol as P

log = logging.getLogger("distrain_b200.data")


def write_shard(path: str, tokens) -> int:
    arr = np.asarray(tokens, dtype="<u2")
    arr.tofile(path)
    return arr.size


def write_manifest(out_dir: str, shard_files: List[str], vocab_size: int) -> dict:
    shards = []
    total = 0
    for f in shard_files:
        n = os.path.getsize(os.path.join(out_dir, f)) // 2
        shards.append({"filename": f, "num_tokens": n, "size_bytes": n * 2})
        total += n
    m = {"num_shards": len(shards), "vocab_size": vocab_size, "shards": shards, "total_tokens": total}
    with open(os.path.join(out_dir, "manifest.json"), "w") as fh:
        json.dump(m, fh, indent=2)
    return m


def prepare_random_shards(out_dir: str, num_shards: int, tokens_per_shard: int, vocab_size: int, seed: int = 0):
    """The data-prep script's ``test`` mode: uniform-random token shards (prepare_data.py:175-186)."""
    os.makedirs(out_dir, exist_ok=True)
    rng = np.random.default_rng(seed)
    files = []
    for i in range(num_shards):
        f = f"shard_{i:04d}.bin"
        write_shard(os.path.join(out_dir, f), rng.integers(0, vocab_size, tokens_per_shard, dtype=np.uint16))
        files.append(f)
    return write_manifest(out_dir, files, vocab_size)


def iter_text_documents(paths: List[str], text_column: str = "text", max_docs: Optional[int] = None):
    """Documents of local files: ``.jsonl`` (one JSON object per line, its ``text_column`` field),
    ``.parquet`` (the ``text_column`` column, read in record batches) or plain text (one document per
    non-empty line)."""
    n = 0
    for path in paths:
        if path.endswith(".parquet"):
            import pyarrow.parquet as pq
            pf = pq.ParquetFile(path)
            for rb in pf.iter_batches(columns=[text_column], batch_size=1024):
                for t in rb.column(0).to_pylist():
                    if max_docs is not None and n >= max_docs:
                        return
                    n += 1
                    yield t or ""
            continue
        with open(path, encoding="utf-8") as fh:
            for line in fh:
                if max_docs is not None and n >= max_docs:
                    return
                if path.endswith(".jsonl") or path.endswith(".json"):
                    line = line.strip()
                    if not line:
                        continue
                    t = json.loads(line).get(text_column, "")
                else:
                    t = line.rstrip("\n")
                n += 1
                yield t


def tokenize_to_shards(texts, out_dir: str, tokenizer_path: str, vocab_size: Optional[int] = None,
                       tokens_per_shard: int = 10_000_000, batch_docs: int = 1000) -> dict:
    """Tokenize documents (an iterable of strings) into ``shard_XXXX.bin`` files of ``tokens_per_shard``
    uint16 ids and write the manifest (reference scripts/prepare_data.py:106-167).

    Empty documents are skipped; documents are encoded in batches and their ids concatenated without
    separators; every full shard is written as it fills; the remainder becomes a final shard only when it
    holds at least a tenth of a shard, otherwise it is dropped. The tokenizer's vocabulary must fit
    uint16 and, when ``vocab_size`` is given, match it (the model's embedding size)."""
    from tokenizers import Tokenizer
    tok = Tokenizer.from_file(tokenizer_path)
    v = tok.get_vocab_size()
    if v > 65536:
        raise ValueError(f"tokenizer vocabulary {v} does not fit uint16 token ids")
    if vocab_size is not None and v != vocab_size:
        raise ValueError(f"tokenizer vocabulary {v} != model vocabulary {vocab_size}")
    os.makedirs(out_dir, exist_ok=True)
    files: List[str] = []
    buf = np.empty(0, dtype=np.uint16)
    dropped = 0

    def emit(arr):
        f = f"shard_{len(files):04d}.bin"
        write_shard(os.path.join(out_dir, f), arr)
        files.append(f)

    def encode(batch):
        nonlocal buf
        ids = [np.asarray(e.ids, dtype=np.uint16) for e in tok.encode_batch(batch)]
        buf = np.concatenate([buf] + ids) if ids else buf
        while buf.size >= tokens_per_shard:
            emit(buf[:tokens_per_shard])
            buf = buf[tokens_per_shard:]

    batch: List[str] = []
    for t in texts:
        if not t or not t.strip():
            continue
        batch.append(t)
        if len(batch) >= batch_docs:
            encode(batch)
            batch = []
    if batch:
        encode(batch)
    if buf.size and buf.size >= tokens_per_shard // 10:
        emit(buf)
    else:
        dropped = int(buf.size)
    m = write_manifest(out_dir, files, vocab_size if vocab_size is not None else v)
    m["dropped_tail_tokens"] = dropped
    return m


def _reg():
    v, ll, i, ull = ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_ulonglong
    register("dtr_loader_open", [ctypes.c_char_p, ll, ll, i], v)
    register("dtr_loader_total_tokens", [v], ull)
    register("dtr_loader_resident", [v], i)
    register("dtr_loader_position", [v, v], ll)
    register("dtr_loader_next", [v, v, ll], i)
    register("dtr_loader_seek_by_seed", [v, ull], None)
    register("dtr_loader_seek", [v, ll, ll], i)
    register("dtr_loader_reset", [v], None)
    register("dtr_loader_start_prefetch", [v, v, i], i)
    register("dtr_loader_acquire", [v, i], i)
    register("dtr_loader_release", [v, i], None)
    register("dtr_loader_error", [v], ctypes.c_char_p)
    register("dtr_loader_close", [v], None)


class ShardLoader:
    def __init__(self, paths: List[str], seq_len: int, batch_size: int, max_resident: int = 0,
                 prefetch: int = 0, pin: bool = True):
        _reg()
        self.L = rt()
        self.seq_len, self.batch_size = seq_len, batch_size
        self.h = self.L.dtr_loader_open("\n".join(paths).encode(), seq_len, batch_size, max_resident)
        if not self.h:
            raise NativeError(f"cannot open shards (missing file or fewer than {seq_len * batch_size} tokens)")
        self.bufs = None
        if prefetch:
            mk = (lambda: torch.empty(batch_size, seq_len, dtype=torch.int32).pin_memory()) if pin and \
                torch.cuda.is_available() else (lambda: torch.empty(batch_size, seq_len, dtype=torch.int32))
            self.bufs = [mk() for _ in range(prefetch)]
            arr = (ctypes.c_void_p * prefetch)(*[b.data_ptr() for b in self.bufs])
            self._arr = arr
            if self.L.dtr_loader_start_prefetch(self.h, arr, prefetch):
                raise NativeError("prefetch start failed")
        self._held = None

    @property
    def total_tokens(self) -> int:
        return int(self.L.dtr_loader_total_tokens(self.h))

    def next_batch(self, batch_size: Optional[int] = None) -> torch.Tensor:
        """[batch, seq_len] int32. With prefetch the returned tensor is a pinned slot that stays valid until
        the next call."""
        if self.bufs is not None:
            if self._held is not None:
                self.L.dtr_loader_release(self.h, self._held)
            s = self.L.dtr_loader_acquire(self.h, 60000)
            if s < 0:
                raise NativeError(f"prefetch failed: {self.L.dtr_loader_error(self.h).decode()}")
            self._held = s
            return self.bufs[s]
        bs = batch_size or self.batch_size
        out = torch.empty(bs, self.seq_len, dtype=torch.int32)
        if self.L.dtr_loader_next(self.h, out.data_ptr(), bs):
            raise NativeError(self.L.dtr_loader_error(self.h).decode())
        return out

    def seek_by_seed(self, seed: int):
        self.L.dtr_loader_seek_by_seed(self.h, seed)

    def reset(self):
        self.L.dtr_loader_reset(self.h)

    def state(self):
        """The read position (shard, token offset), or None while prefetching (the prefetch thread reads
        ahead of the batches handed out, so its position is not the consumer's)."""
        if self.bufs is not None:
            return None
        shard, off = self.position()
        return {"shard": shard, "offset": off}

    def restore(self, st):
        """Continue from a position saved by ``state``."""
        rc = self.L.dtr_loader_seek(self.h, int(st["shard"]), int(st["offset"]))
        if rc:
            raise NativeError(f"cannot seek to {st} (rc {rc})")

    def position(self):
        off = ctypes.c_longlong(0)
        return int(self.L.dtr_loader_position(self.h, ctypes.byref(off))), int(off.value)

    def resident_shards(self) -> int:
        return int(self.L.dtr_loader_resident(self.h))

    def close(self):
        if self.h:
            self.L.dtr_loader_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class StreamingLoader:
    """Assigned shards from an object store (key layout data/shard_XXXX.bin), cached locally."""

    def __init__(self, store, cache_dir: str, shard_indices: List[int], seq_len: int, batch_size: int,
                 max_resident: int = 4, prefetch: int = 2):
        os.makedirs(cache_dir, exist_ok=True)
        manifest = store.get_json(P.manifest_path())
        paths, self.skipped = [], []
        for i in shard_indices:
            entry = manifest["shards"][i]
            local = os.path.join(cache_dir, entry["filename"])
            if not os.path.exists(local):
                try:
                    store.download_to_file(f"data/{entry['filename']}", local)
                except Exception as e:  # a shard that cannot be fetched is skipped (reference data.rs:392-395)
                    self.skipped.append((entry["filename"], str(e)))
                    continue
            paths.append(local)
        if not paths:
            raise NativeError(f"none of the assigned shards could be fetched: {self.skipped[:3]}")
        self.manifest = manifest
        self.files = [os.path.basename(p) for p in paths]
        self.loader = ShardLoader(paths, seq_len, batch_size, max_resident=max_resident, prefetch=prefetch)

    def next_batch(self):
        return self.loader.next_batch()

    def state(self):
        """The read position with the shard's file name: the loaded shard list depends on which shards
        could be fetched, so an index alone would point elsewhere after a restart that fetched others."""
        st = self.loader.state()
        if st is not None:
            st = dict(st, filename=self.files[st["shard"]])
        return st

    def restore(self, st):
        """Continue from ``state``: the saved shard is found by file name. When that shard was not fetched
        this time, reading restarts at the first loaded shard (the position cannot be mapped)."""
        st = dict(st)
        name = st.get("filename")
        if name is not None:
            if name not in self.files:
                log.warning("saved data position is in shard %s, which was not fetched; starting over", name)
                st["shard"], st["offset"] = 0, 0
            else:
                st["shard"] = self.files.index(name)
        self.loader.restore(st)

    def close(self):
        self.loader.close()


class SyntheticTokens:
    """Seeded uniform-random token ids in [0, vocab) (the benchmark's synthetic data)."""

    def __init__(self, vocab: int, batch: int, seq_len: int, seed: int):
        self.g = torch.Generator().manual_seed(seed)
        self.vocab, self.batch, self.seq_len = vocab, batch, seq_len

    def next_batch(self) -> torch.Tensor:
        return torch.randint(0, self.vocab, (self.batch, self.seq_len), generator=self.g, dtype=torch.int32)

    def state(self):
        return {"generator": self.g.get_state()}

    def restore(self, st):
        self.g.set_state(st["generator"])
