"""The C ABI of libdistrain_c.so (csrc/ffi/distrain_c.h) on the CPU backend:

* called in-process through ctypes: training steps give exactly the losses of the engine driven from
  Python on the same weights and batches (so the optimizer keeps its state across calls), checkpoint
  loading infers the model and installs its weights, the delta file decodes to the compressed
  snapshot - current difference, failures come back as {"error": ...}, and the native helpers (shard
  assignment, cosine schedule) agree with the Python ones;
* called from a C program that links the library, which then starts its own interpreter."""
import ctypes
import json
import os
import shutil
import subprocess

import pytest
import torch

from distrain_b200 import _build
from distrain_b200.config import CompressionConfig, OptimConfig, TrainingParams, cosine_lr, preset
from distrain_b200.models import oracle
from distrain_b200.models.params import ParamLayout, init_flat
from distrain_b200.parallel.compression import compress_reference
from distrain_b200.parallel.http_node import CpuBackend
from distrain_b200.utils.checkpoint import save_safetensors
from distrain_b200.utils.data import ShardLoader, prepare_random_shards
from distrain_b200.utils.delta_codec import decode_delta
from distrain_b200.utils.native import shard_assignment

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    path = _build.build_ffi()
    L = ctypes.CDLL(path)
    vp, cp = ctypes.c_void_p, ctypes.c_char_p
    for name, args in (("distrain_init", [cp]), ("distrain_load_shards", [cp, ctypes.c_size_t, ctypes.c_size_t]),
                       ("distrain_train_step", [ctypes.c_double]), ("distrain_status", []),
                       ("distrain_calibrate", [ctypes.c_double]), ("distrain_load_checkpoint_file", [cp]),
                       ("distrain_load_checkpoint", [vp, ctypes.c_size_t]), ("distrain_snapshot_params", []),
                       ("distrain_compute_delta", [cp]), ("distrain_default_training_params", []),
                       ("distrain_compute_shard_assignment", [cp, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32])):
        f = getattr(L, name)
        f.argtypes, f.restype = args, vp
    L.distrain_free_string.argtypes = [vp]
    L.distrain_set_backend.argtypes = [ctypes.c_uint8]
    L.distrain_cosine_lr.argtypes = [ctypes.c_uint64] * 3 + [ctypes.c_double] * 2
    L.distrain_cosine_lr.restype = ctypes.c_double
    L.distrain_set_backend(0)
    yield L
    L.distrain_shutdown()


def _j(L, ptr):
    s = ctypes.cast(ptr, ctypes.c_char_p).value.decode()
    L.distrain_free_string(ptr)
    return json.loads(s)


@pytest.fixture(scope="module")
def shards(tmp_path_factory):
    d = tmp_path_factory.mktemp("shards")
    prepare_random_shards(str(d), 2, 40_000, 256, seed=3)
    return [str(d / f"shard_{i:04d}.bin") for i in range(2)]


def test_steps_match_the_python_engine(lib, shards, tmp_path):
    st = _j(lib, lib.distrain_init(b"MicroTest"))
    assert st == {"initialized": True, "step": 0, "last_loss": 0.0, "total_tokens": 0, "model_preset": "MicroTest",
                  "gpu": False}
    assert _j(lib, lib.distrain_load_shards(json.dumps(shards).encode(), 2, 32)) == {"ok": True, "shards": 2}
    assert _j(lib, lib.distrain_snapshot_params())["num_params"] == ParamLayout(preset("micro")).num_params()
    got = [_j(lib, lib.distrain_train_step(ctypes.c_double(lr))) for lr in (1e-3, 5e-4, 2e-4)]
    assert [g["step"] for g in got] == [1, 2, 3] and got[-1]["tokens_processed"] == 3 * 64
    # the same three steps from Python: same init, same batches, one optimizer across the steps
    cfg = preset("micro")
    L = ParamLayout(cfg)
    b = CpuBackend(cfg, OptimConfig())
    sd0 = L.to_state_dict(init_flat(L, 0.02, 0))
    b.load(sd0)
    src = ShardLoader(shards, 32, 2)
    want = [b.step(src.next_batch(), lr) for lr in (1e-3, 5e-4, 2e-4)]
    assert [g["loss"] for g in got] == pytest.approx(want, rel=1e-6, abs=1e-6)
    # the delta file: the snapshot - current difference through error feedback, top-k and INT8
    out = tmp_path / "d.delta.zst"
    assert _j(lib, lib.distrain_compute_delta(str(out).encode()))["size_bytes"] == out.stat().st_size
    dec = decode_delta(out.read_bytes())
    cur = b.state()
    delta = {k: sd0[k] - cur[k] for k in sd0}
    ref, _ = compress_reference(delta, {k: list(v.shape) for k, v in cur.items()}, CompressionConfig(int8_block=0), {})
    for k in sd0:
        dense = torch.zeros(delta[k].numel())
        dense[ref.indices[k].long()] = ref.values[k]
        assert torch.allclose(dec[k].reshape(-1), dense, rtol=1e-6, atol=1e-9), k
        assert 0 < len(ref.indices[k]) < delta[k].numel() or delta[k].numel() < 100
    s = _j(lib, lib.distrain_status())
    assert (s["step"], s["total_tokens"], s["last_loss"]) == (3, 192, got[-1]["loss"])


def test_checkpoint_load_installs_the_weights(lib, shards, tmp_path):
    cfg = preset("micro")
    L = ParamLayout(cfg)
    sd = L.to_state_dict(init_flat(L, 0.05, 7))
    blob = save_safetensors(sd)
    buf = ctypes.create_string_buffer(blob, len(blob))
    r = _j(lib, lib.distrain_load_checkpoint(ctypes.cast(buf, ctypes.c_void_p), len(blob)))
    assert r["ok"] and r["num_params"] == L.num_params() and r["gpu"] is False
    assert _j(lib, lib.distrain_load_shards(json.dumps(shards).encode(), 2, 32))["ok"]
    first = _j(lib, lib.distrain_train_step(ctypes.c_double(0.0)))["loss"]
    want = float(oracle.lm_loss({k: v.float() for k, v in sd.items()}, cfg, ShardLoader(shards, 32, 2).next_batch().long()))
    assert first == pytest.approx(want, rel=1e-5)
    path = tmp_path / "ck.safetensors"
    path.write_bytes(blob)
    assert _j(lib, lib.distrain_load_checkpoint_file(str(path).encode()))["num_params"] == L.num_params()
    assert _j(lib, lib.distrain_status())["model_preset"] == "checkpoint"


def test_errors_come_back_as_json(lib):
    assert "unknown preset" in _j(lib, lib.distrain_init(b"Huge"))["error"]
    assert "error" in _j(lib, lib.distrain_load_checkpoint(None, 0))
    assert "error" in _j(lib, lib.distrain_load_shards(b"not json", 2, 32))
    assert "No such file" in _j(lib, lib.distrain_load_checkpoint_file(b"/nonexistent/ck.safetensors"))["error"]
    _j(lib, lib.distrain_init(b"micro"))
    assert "snapshot" in _j(lib, lib.distrain_compute_delta(b"/tmp/never-written.delta.zst"))["error"]


def test_native_helpers_and_calibration(lib):
    assert _j(lib, lib.distrain_compute_shard_assignment(b"node-7", 4, 30, 5)) == shard_assignment("node-7", 4, 30, 5)
    for step in (0, 5, 10, 60, 110, 200):
        assert lib.distrain_cosine_lr(step, 10, 110, 3e-4, 1e-6) == pytest.approx(cosine_lr(step, 10, 110, 3e-4, 1e-6),
                                                                                 rel=1e-12, abs=1e-15)
    assert _j(lib, lib.distrain_default_training_params()) == TrainingParams().to_dict()
    c = _j(lib, lib.distrain_calibrate(ctypes.c_double(30.0)))
    assert c["secs_per_step"] > 0 and 5 <= c["recommended_h_mini"] <= 1000


C_PROGRAM = r"""
#include <stdio.h>
#include "distrain_c.h"
static void show(char* r) { printf("%s\n", r); distrain_free_string(r); }
int main(int argc, char** argv) {
  distrain_set_backend(0);
  show(distrain_init("MicroTest"));
  show(distrain_load_shards(argv[1], 2, 32));
  show(distrain_snapshot_params());
  for (int i = 0; i < 2; ++i) show(distrain_train_step(1e-3));
  show(distrain_compute_delta(argv[2]));
  distrain_shutdown();
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_a_c_program_starts_its_own_interpreter(shards, tmp_path):
    so = _build.build_ffi()
    src = tmp_path / "main.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "main"
    libdir = os.path.dirname(so)
    subprocess.run(["gcc", "-O1", "-I", os.path.join(ROOT, "csrc", "ffi"), str(src), "-o", str(exe), "-L", libdir,
                    "-ldistrain_c", f"-Wl,-rpath,{libdir}"], check=True)
    env = {k: v for k, v in os.environ.items() if k not in ("PYTHONPATH", "PYTHONHOME")}
    r = subprocess.run([str(exe), json.dumps(shards), str(tmp_path / "c.delta.zst")], capture_output=True, text=True,
                       timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
    assert lines[0]["initialized"] and lines[1] == {"ok": True, "shards": 2}
    assert [x["step"] for x in lines[3:5]] == [1, 2] and lines[5]["ok"]
    assert decode_delta((tmp_path / "c.delta.zst").read_bytes())


def test_config_inference_recovers_every_preset():
    """Checkpoint shapes -> model config: the head split of each preset comes back (shapes alone would
    allow others), and a vocabulary that differs from the preset's is taken from the checkpoint."""
    from distrain_b200.cli import _infer_model_config
    for name in ("micro", "tiny", "small", "medium", "large"):
        cfg = preset(name)
        for vocab in (cfg.vocab_size, 32768 + 64):
            cfg.vocab_size = vocab
            sd = {e.name: torch.empty(e.shape, device="meta") for e in ParamLayout(cfg).entries}
            got = _infer_model_config(sd)
            assert (got.num_heads, got.num_kv_heads, got.hidden_dim, got.num_layers, got.ffn_hidden_dim,
                    got.vocab_size) == (cfg.num_heads, cfg.num_kv_heads, cfg.hidden_dim, cfg.num_layers,
                                        cfg.ffn_hidden_dim, vocab), name
