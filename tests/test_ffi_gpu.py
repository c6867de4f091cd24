"""The C ABI of libdistrain_c.so (csrc/ffi/distrain_c.h) on the CUDA backend: distrain_train_step drives
the sm_100a training engine, its losses equal those of the same engine driven from Python on the same
initial weights and batches (the engine, and its AdamW state, persist across calls), and the status
reports the GPU backend; the delta file decodes to the snapshot - current difference."""
import ctypes
import json

import pytest
import torch

from distrain_b200 import _build
from distrain_b200.config import OptimConfig, preset
from distrain_b200.models.params import ParamLayout, init_flat
from distrain_b200.parallel.http_node import CudaBackend
from distrain_b200.utils.data import ShardLoader, prepare_random_shards
from distrain_b200.utils.delta_codec import decode_delta

pytestmark = pytest.mark.gpu


def _j(L, ptr):
    s = ctypes.cast(ptr, ctypes.c_char_p).value.decode()
    L.distrain_free_string(ptr)
    return json.loads(s)


def test_train_steps_on_the_cuda_engine(tmp_path):
    L = ctypes.CDLL(_build.build_ffi())
    vp, cp = ctypes.c_void_p, ctypes.c_char_p
    for name, args in (("distrain_init", [cp]), ("distrain_load_shards", [cp, ctypes.c_size_t, ctypes.c_size_t]),
                       ("distrain_train_step", [ctypes.c_double]), ("distrain_status", []),
                       ("distrain_snapshot_params", []), ("distrain_compute_delta", [cp])):
        f = getattr(L, name)
        f.argtypes, f.restype = args, vp
    L.distrain_free_string.argtypes = [vp]
    L.distrain_set_backend.argtypes = [ctypes.c_uint8]
    L.distrain_set_backend.restype = None
    L.distrain_set_backend(1)
    prepare_random_shards(str(tmp_path), 2, 40_000, 256, seed=4)
    shards = [str(tmp_path / f"shard_{i:04d}.bin") for i in range(2)]
    try:
        st = _j(L, L.distrain_init(b"MicroTest"))
        assert st["gpu"] is True
        assert _j(L, L.distrain_load_shards(json.dumps(shards).encode(), 4, 65))["ok"]
        assert _j(L, L.distrain_snapshot_params())["num_params"] == ParamLayout(preset("micro")).num_params()
        got = [_j(L, L.distrain_train_step(ctypes.c_double(lr))) for lr in (1e-3, 5e-4, 2e-4)]
        assert [g["step"] for g in got] == [1, 2, 3] and got[-1]["tokens_processed"] == 3 * 4 * 65
        # the same steps driven from Python on the same engine type, weights and batches
        cfg = preset("micro")
        cfg.max_seq_len = max(cfg.max_seq_len, 65)
        lay = ParamLayout(cfg)
        b = CudaBackend(cfg, OptimConfig(), 4, 65, torch.device("cuda", 0))
        b.load(lay.to_state_dict(init_flat(lay, 0.02, 0)))
        src = ShardLoader(shards, 65, 4)
        want = [b.step(src.next_batch(), lr) for lr in (1e-3, 5e-4, 2e-4)]
        assert [g["loss"] for g in got] == pytest.approx(want, rel=1e-3, abs=1e-3)
        assert want[-1] < want[0] + 1.0
        s = _j(L, L.distrain_status())
        assert s["gpu"] is True and s["step"] == 3
        out = tmp_path / "d.delta.zst"
        assert _j(L, L.distrain_compute_delta(str(out).encode()))["size_bytes"] == out.stat().st_size
        dec = decode_delta(out.read_bytes())
        assert set(dec) == {e.name for e in lay.entries}
        assert sum(int((t != 0).sum()) for t in dec.values()) > 0
    finally:
        L.distrain_shutdown()
