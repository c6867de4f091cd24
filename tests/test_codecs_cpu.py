"""Native runtime codecs: safetensors, zstd, reference SparseDelta JSON, DTZ1, shard assignment."""
import json
import math
import struct

import torch

from distrain_b200.utils import native
from distrain_b200.utils.checkpoint import save_safetensors, load_safetensors, load_safetensors_bytes, \
    save_velocity, load_velocity
from distrain_b200.utils.delta_codec import encode_sparse_delta, decode_delta, encode_dtz, decode_dtz_dense, \
    LowRankPayload
from distrain_b200.parallel.compression import compress_reference, reconstruct_dense, quantize_int8, \
    dequantize_int8, sparsify_topk
from distrain_b200.config import CompressionConfig


def test_safetensors_roundtrip(tmp_path):
    t = {"b.weight": torch.randn(3, 4), "a": torch.randn(7), "scalar": torch.tensor([2.5])}
    p = str(tmp_path / "m.safetensors")
    save_safetensors(t, p)
    back = load_safetensors(p)
    assert set(back) == set(t)
    for k in t:
        assert torch.equal(back[k], t[k])
    raw = save_safetensors(t)
    assert load_safetensors_bytes(raw)["a"].equal(t["a"])
    # header: 8-byte LE length, JSON padded to a multiple of 8, sorted names
    hl = struct.unpack("<Q", raw[:8])[0]
    assert hl % 8 == 0
    hdr = json.loads(raw[8:8 + hl])
    assert hdr["a"]["dtype"] == "F32" and hdr["b.weight"]["shape"] == [3, 4]


def test_safetensors_reads_bf16_f16_written_by_safetensors_pkg(tmp_path):
    from safetensors.torch import save_file
    t = {"x": torch.randn(5, 3).bfloat16(), "y": torch.randn(4).half(), "z": torch.tensor([1e-6, -2.0]).half()}
    p = str(tmp_path / "h.safetensors")
    save_file(t, p)
    back = load_safetensors(p)
    for k in t:
        assert torch.equal(back[k], t[k].float())


def test_velocity_file_layout(tmp_path):
    v = {"w": torch.randn(2, 3)}
    raw = save_velocity(v)
    sd = load_safetensors_bytes(raw)
    assert list(sd) == ["velocity.w"] and sd["velocity.w"].shape == (6,)
    assert torch.equal(load_velocity(raw)["w"], v["w"].reshape(-1))


def test_zstd_roundtrip():
    data = b"distrain" * 1000
    c = native.zstd_compress(data, 3)
    assert len(c) < len(data) and c[:4] == b"\x28\xb5\x2f\xfd"
    assert native.zstd_decompress(c) == data


def test_reference_cross_framework_fixture():
    """The reference's Python-produced JSON fixture (core/model/src/compression.rs:631-656)."""
    fixture = json.dumps({
        "indices": {"weight": [0, 5, 10, 50, 99]},
        "values": {"weight": [0.1, -0.3, 0.5, -0.2, 0.4]},
        "shapes": {"weight": [100]},
        "scales": {"weight": 0.003937},
        "config": {"top_k_fraction": 0.05, "quantize_int8": True, "zstd_level": 3, "min_top_k_fraction": 0.001,
                   "max_top_k_fraction": 0.1, "per_tensor_adaptive": False}}).encode()
    rec = decode_delta(native.zstd_compress(fixture, 3))
    w = rec["weight"]
    assert w.numel() == 100
    assert abs(w[0] - 0.1) < 1e-6 and abs(w[5] + 0.3) < 1e-6 and abs(w[10] - 0.5) < 1e-6 and w[1] == 0
    # raw JSON (no zstd) fallback
    assert decode_delta(fixture)["weight"].equal(w)


def test_sparse_delta_schema_and_roundtrip():
    torch.manual_seed(0)
    delta = {"param": torch.sin(torch.arange(1000) / 100.0)}
    cfg = CompressionConfig(top_k_fraction=0.1, quantize_int8=True, per_tensor_adaptive=True)
    ef = {}
    sd, stats = compress_reference(delta, {"param": [1000]}, cfg, ef)
    blob = encode_sparse_delta(sd)
    js = json.loads(native.zstd_decompress(blob))
    assert set(js) == {"indices", "values", "shapes", "scales", "config"}
    assert all(isinstance(i, int) for i in js["indices"]["param"])
    assert all(isinstance(v, float) for v in js["values"]["param"])
    assert isinstance(js["config"]["zstd_level"], int) and isinstance(js["config"]["quantize_int8"], bool)
    rec = decode_delta(blob)["param"]
    nz = int((rec != 0).sum())
    assert 99 <= nz <= 101
    dense = reconstruct_dense(sd)["param"]
    assert torch.allclose(rec, dense)


def test_topk_sorted_and_count():
    d = {"w": torch.randn(1000)}
    _, idx, vals = sparsify_topk(d, 0.1, False)
    assert idx["w"].numel() == 100
    assert torch.all(idx["w"][1:] > idx["w"][:-1])


def test_int8_quant_cosine():
    v = torch.randn(5000)
    q, s = quantize_int8(v, 0)
    d = dequantize_int8(q, s, 0)
    cos = torch.nn.functional.cosine_similarity(v, d, dim=0)
    assert cos > 0.99
    q2, s2 = quantize_int8(v, 256)
    assert s2.numel() == math.ceil(5000 / 256)
    assert torch.nn.functional.cosine_similarity(v, dequantize_int8(q2, s2, 256), dim=0) > 0.999


def test_error_feedback_accumulates():
    cfg = CompressionConfig(top_k_fraction=0.1, quantize_int8=False)
    ef = {}
    compress_reference({"weight": torch.ones(100)}, {"weight": [100]}, cfg, ef)
    assert int((ef["weight"].abs() > 1e-8).sum()) > 0


def test_lowrank_json_detected():
    js = json.dumps({"tensors": {"w": {"u": [1.0, 2.0], "v": [3.0], "m": 2, "n": 1, "rank": 1}}, "rank": 1}).encode()
    out = decode_delta(native.zstd_compress(js))
    assert isinstance(out, LowRankPayload) and out["rank"] == 1


def test_dtz_roundtrip():
    idx = torch.tensor([1, 7, 9, 300], dtype=torch.int32)
    q = torch.tensor([127, -3, 5, -127], dtype=torch.int8)
    sc = torch.tensor([0.5], dtype=torch.float32)
    d = decode_dtz_dense(encode_dtz(400, idx, q, sc, None, 256, zstd_level=3))
    assert d.numel() == 400 and d[1] == 63.5 and d[300] == -63.5 and d[0] == 0


# ─────────────── shard assignment (SipHash-1-3 as Rust's DefaultHasher) ───────────────
def _sip13(data: bytes) -> int:
    M = (1 << 64) - 1
    rotl = lambda x, b: ((x << b) | (x >> (64 - b))) & M
    v0, v1, v2, v3 = 0x736f6d6570736575, 0x646f72616e646f6d, 0x6c7967656e657261, 0x7465646279746573

    def rnd(v0, v1, v2, v3):
        v0 = (v0 + v1) & M; v1 = rotl(v1, 13); v1 ^= v0; v0 = rotl(v0, 32)
        v2 = (v2 + v3) & M; v3 = rotl(v3, 16); v3 ^= v2
        v0 = (v0 + v3) & M; v3 = rotl(v3, 21); v3 ^= v0
        v2 = (v2 + v1) & M; v1 = rotl(v1, 17); v1 ^= v2; v2 = rotl(v2, 32)
        return v0, v1, v2, v3

    n = len(data)
    full = n // 8 * 8
    for i in range(0, full, 8):
        m = int.from_bytes(data[i:i + 8], "little")
        v3 ^= m
        v0, v1, v2, v3 = rnd(v0, v1, v2, v3)
        v0 ^= m
    b = ((n & 0xff) << 56) | int.from_bytes(data[full:], "little")
    v3 ^= b
    v0, v1, v2, v3 = rnd(v0, v1, v2, v3)
    v0 ^= b
    v2 ^= 0xff
    for _ in range(3):
        v0, v1, v2, v3 = rnd(v0, v1, v2, v3)
    return v0 ^ v1 ^ v2 ^ v3


def test_siphash13_native_matches_python():
    for s in [b"", b"a", b"12345678", b"0:node-abc", b"x" * 37]:
        assert native.rt().dtr_siphash13(s, len(s)) == _sip13(s)
    assert native.rt().dtr_hash_str(b"3:n1") == _sip13(b"3:n1" + b"\xff")
    assert native.rt().dtr_hash_u64(7) == _sip13((7).to_bytes(8, "little"))


def test_shard_assignment_properties():
    a = native.shard_assignment("node-1", 3, 100, 20)
    assert a == native.shard_assignment("node-1", 3, 100, 20)
    assert len(a) == 20 and len(set(a)) == 20 and all(0 <= x < 100 for x in a)
    assert a != native.shard_assignment("node-2", 3, 100, 20)
    assert a != native.shard_assignment("node-1", 4, 100, 20)
    assert len(native.shard_assignment("n", 0, 5, 50)) == 5
