"""Data loading: shard format, sequential wrap-around batches, seek_by_seed, resident window, prefetch,
streaming from a store (restates the reference's data_tests.rs regressions: no repeats, advancing
position, full coverage)."""
import json
import os

import numpy as np
import pytest
import torch

from distrain_b200.utils.data import ShardLoader, StreamingLoader, prepare_random_shards, write_shard
from distrain_b200.utils.storage import FsStore


def _shards(tmp_path, n=3, size=1000):
    paths = []
    for i in range(n):
        p = str(tmp_path / f"shard_{i:04d}.bin")
        write_shard(p, np.arange(i * size, (i + 1) * size) % 65536)
        paths.append(p)
    return paths


def test_sequential_batches_wrap_and_no_repeat(tmp_path):
    paths = _shards(tmp_path)
    L = ShardLoader(paths, seq_len=10, batch_size=4)
    seen = []
    for _ in range(75):  # 3000 tokens = exactly all shards once
        b = L.next_batch()
        assert b.shape == (4, 10) and b.dtype == torch.int32
        seen.append(b.reshape(-1))
    allt = torch.cat(seen)
    assert torch.equal(allt, torch.arange(3000, dtype=torch.int32))   # full coverage, no repeats, in order
    assert L.next_batch()[0, 0].item() == 0                            # wraps around
    L.close()


def test_batch_spans_shard_boundary(tmp_path):
    paths = _shards(tmp_path, n=2, size=25)
    L = ShardLoader(paths, seq_len=10, batch_size=3)
    b = L.next_batch()
    assert b.reshape(-1).tolist() == list(range(30))


def test_seek_by_seed_matches_reference_formula(tmp_path):
    paths = _shards(tmp_path, n=3, size=1000)
    L = ShardLoader(paths, seq_len=16, batch_size=1)
    for seed in (0, 1, 7, 12345):
        L.seek_by_seed(seed)
        si = seed % 3
        pos = ((seed * 0x9E3779B97F4A7C15) % (1 << 64)) % 1000
        off = pos // 16 * 16
        assert L.position() == (si, off)
        assert L.next_batch()[0, 0].item() == si * 1000 + off


def test_resident_window_bounded(tmp_path):
    paths = _shards(tmp_path, n=5, size=100)
    L = ShardLoader(paths, seq_len=10, batch_size=10, max_resident=2)
    for _ in range(7):
        L.next_batch()
        assert L.resident_shards() <= 2


def test_prefetch_matches_sync(tmp_path):
    paths = _shards(tmp_path, n=2, size=500)
    a = ShardLoader(paths, seq_len=8, batch_size=4)
    b = ShardLoader(paths, seq_len=8, batch_size=4, prefetch=3, pin=False)
    for _ in range(40):
        assert torch.equal(a.next_batch(), b.next_batch())
    b.close()


def test_prepare_and_stream_from_store(tmp_path):
    src = str(tmp_path / "prep")
    m = prepare_random_shards(src, num_shards=4, tokens_per_shard=2048, vocab_size=300, seed=1)
    assert m["num_shards"] == 4 and m["total_tokens"] == 8192 and m["vocab_size"] == 300
    store = FsStore(str(tmp_path / "obj"))
    for f in os.listdir(src):
        store.upload_from_file(os.path.join(src, f), f"data/{f}")
    s = StreamingLoader(store, str(tmp_path / "cache"), [2, 0], seq_len=64, batch_size=2, prefetch=2)
    b = s.next_batch()
    ref = np.fromfile(os.path.join(src, "shard_0002.bin"), dtype="<u2")[:128].astype(np.int32)
    assert torch.equal(b.reshape(-1), torch.from_numpy(ref)) and int(b.max()) < 300
    s.close()


def test_stream_skips_a_shard_that_cannot_be_fetched(tmp_path):
    src = str(tmp_path / "prep")
    prepare_random_shards(src, num_shards=3, tokens_per_shard=2048, vocab_size=300, seed=2)
    store = FsStore(str(tmp_path / "obj"))
    for f in os.listdir(src):
        if f != "shard_0001.bin":  # listed in the manifest, missing from the store
            store.upload_from_file(os.path.join(src, f), f"data/{f}")
    s = StreamingLoader(store, str(tmp_path / "cache"), [1, 2], seq_len=64, batch_size=2, prefetch=0)
    assert [f for f, _ in s.skipped] == ["shard_0001.bin"]
    ref = np.fromfile(os.path.join(src, "shard_0002.bin"), dtype="<u2")[:128].astype(np.int32)
    assert torch.equal(s.next_batch().reshape(-1), torch.from_numpy(ref))
    s.close()
    with pytest.raises(Exception):
        StreamingLoader(store, str(tmp_path / "cache2"), [1], seq_len=64, batch_size=2)


def test_stream_resume_maps_the_position_by_shard_name(tmp_path):
    """A position saved while a shard was unavailable resumes in the same shard file once that shard can be
    fetched again (the loaded shard list, and so the shard index, differs between the two runs)."""
    src = str(tmp_path / "prep")
    prepare_random_shards(src, num_shards=3, tokens_per_shard=2048, vocab_size=300, seed=3)
    store = FsStore(str(tmp_path / "obj"))
    for f in os.listdir(src):
        if f != "shard_0001.bin":
            store.upload_from_file(os.path.join(src, f), f"data/{f}")
    s = StreamingLoader(store, str(tmp_path / "cache"), [1, 2], seq_len=64, batch_size=2, prefetch=0)
    for _ in range(3):
        s.next_batch()
    st = s.state()
    assert st["filename"] == "shard_0002.bin" and st["shard"] == 0
    expect = s.next_batch()
    s.close()
    store.upload_from_file(os.path.join(src, "shard_0001.bin"), "data/shard_0001.bin")
    s2 = StreamingLoader(store, str(tmp_path / "cache2"), [1, 2], seq_len=64, batch_size=2, prefetch=0)
    assert s2.files == ["shard_0001.bin", "shard_0002.bin"]
    s2.restore(st)
    assert torch.equal(s2.next_batch(), expect)
    s2.close()


def _word_tokenizer(tmp_path, words):
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import Whitespace
    vocab = {"[UNK]": 0}
    for w in words:
        vocab.setdefault(w, len(vocab))
    tok = Tokenizer(WordLevel(vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = Whitespace()
    path = str(tmp_path / "tok.json")
    tok.save(path)
    return path, tok, len(vocab)


def test_tokenize_to_shards_from_text_jsonl_and_parquet(tmp_path):
    """Documents from .txt, .jsonl and .parquet inputs are encoded in order, concatenated and cut into
    full shards; a remainder of at least a tenth of a shard becomes the final shard."""
    import pyarrow as pa
    import pyarrow.parquet as pq
    from distrain_b200.utils.data import iter_text_documents, tokenize_to_shards
    from distrain_b200 import cli
    words = [f"w{i}" for i in range(50)]
    tok_path, tok, V = _word_tokenizer(tmp_path, words)
    rng = np.random.default_rng(0)
    docs = [" ".join(rng.choice(words, size=int(rng.integers(3, 30)))) for _ in range(120)]
    (tmp_path / "a.txt").write_text("\n".join(docs[:40]) + "\n\n")
    with open(tmp_path / "b.jsonl", "w") as fh:
        for d in docs[40:80]:
            fh.write(json.dumps({"text": d, "id": 1}) + "\n")
    pq.write_table(pa.table({"text": docs[80:]}), str(tmp_path / "c.parquet"))
    inputs = [str(tmp_path / f) for f in ("a.txt", "b.jsonl", "c.parquet")]
    got = list(iter_text_documents(inputs))
    assert [g for g in got if g] == docs
    want = np.concatenate([np.asarray(tok.encode(d).ids, dtype=np.uint16) for d in docs])
    per = 300
    m = tokenize_to_shards(iter_text_documents(inputs), str(tmp_path / "out"), tok_path, V, per, batch_docs=7)
    full = want.size // per
    rem = want.size - full * per
    assert m["num_shards"] == full + (1 if rem >= per // 10 else 0) and m["vocab_size"] == V
    back = np.concatenate([np.fromfile(str(tmp_path / "out" / s["filename"]), dtype="<u2") for s in m["shards"]])
    assert np.array_equal(back, want[:back.size]) and back.size in (want.size, full * per)
    with pytest.raises(ValueError):
        tokenize_to_shards(docs, str(tmp_path / "bad"), tok_path, V + 1, per)
    # the CLI entry point
    cli.main(["prepare-data", "--output-dir", str(tmp_path / "cli"), "--input", inputs[1], "--tokenizer", tok_path,
              "--vocab", str(V), "--tokens-per-shard", "100"])
    assert json.load(open(tmp_path / "cli" / "manifest.json"))["num_shards"] >= 1
