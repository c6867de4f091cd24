"""An HTTP node training on a B200 compresses its round deltas on the device: the exact per-tensor top-k
with error feedback runs in the sm_100a compression kernels and only the kept (index, value) pairs cross
to the host; the decoded push equals the reference compression of the same round delta."""
import threading

import pytest
import torch

from distrain_b200.config import CompressionConfig, CoordinatorConfig, ModelConfig, OptimConfig
from distrain_b200.coordinator.service import CoordinatorService, bootstrap
from distrain_b200.models.params import ParamLayout, init_flat
from distrain_b200.parallel.compression import compress_reference
from distrain_b200.parallel.http_node import CudaBackend, HttpNode
from distrain_b200.utils.storage import FsStore

pytestmark = pytest.mark.gpu

CFG = ModelConfig(hidden_dim=128, num_layers=2, num_heads=2, num_kv_heads=1, ffn_hidden_dim=256, vocab_size=512,
                  max_seq_len=128, rope_theta=10000.0)


@pytest.mark.parametrize("quant", [False, True])
def test_device_round_delta_matches_reference_compression(quant):
    torch.manual_seed(0)
    comp = CompressionConfig(top_k_fraction=0.1, quantize_int8=quant, per_tensor_adaptive=True)
    b = CudaBackend(CFG, OptimConfig(lr=3e-3), 4, 65, torch.device("cuda", 0))
    lay = ParamLayout(CFG)
    b.load(lay.to_state_dict(init_flat(lay, 0.02, 1)))
    b.enable_device_compression(comp, 0.1)
    ef = {}
    for rnd in range(2):  # the second round carries the first round's error feedback
        start = b.state()
        for _ in range(3):
            b.step(torch.randint(0, CFG.vocab_size, (4, 65), dtype=torch.int32), 3e-3)
        cur = b.state()
        delta = {k: (start[k] - cur[k]).reshape(-1) for k in start}
        ref, rstats = compress_reference(delta, {k: list(v.shape) for k, v in cur.items()}, comp, ef)
        sd, stats = b.collect(b.compress_round(0.1), comp)
        assert b.d2h_bytes_last == 8 * stats["num_params_kept"]
        assert stats["num_params_kept"] == rstats["num_params_kept"]
        for k in delta:
            assert torch.equal(sd.indices[k].long(), ref.indices[k].long()), k
            assert torch.allclose(sd.values[k], ref.values[k], rtol=1e-6, atol=0), k
            if quant:
                assert sd.scales[k] == pytest.approx(ref.scales[k], rel=1e-6)
        assert stats["dense_norm"] == pytest.approx(rstats["dense_norm"], rel=1e-5)


@pytest.mark.timeout(600)
def test_gpu_http_node_pushes_device_compressed_deltas(tmp_path):
    store = FsStore(str(tmp_path))
    bootstrap(store, CFG, seed=0)
    svc = CoordinatorService(CoordinatorConfig(min_contributions=0), store, flush_interval=3600)
    port = svc.start(host="127.0.0.1", port=0, threads=4)
    url = f"http://127.0.0.1:{port}"
    g = torch.Generator().manual_seed(5)
    pool = torch.randint(0, CFG.vocab_size, (8, 65), generator=g, dtype=torch.int32)
    data = lambda: pool[torch.randint(0, 8, (4,), generator=g)]
    n = HttpNode(url, store, CFG, batch=4, seq_len=65, h_mini=5, optim=OptimConfig(lr=3e-3),
                 compression=CompressionConfig(top_k_fraction=0.1, quantize_int8=True), device="cuda",
                 node_id="gpu-node", data=data, poll_secs=0.2)
    assert n.device_comp
    n.register()
    t = threading.Thread(target=n.run, args=(40,))
    t.start()
    t.join()
    svc.stop()
    assert not svc.last_error, svc.last_error
    assert not n.errors, n.errors
    assert any(p["accepted"] for p in n.pushes)
    assert svc.acc.state.checkpoint_version >= 1
    kept = max(p["bytes"] for p in n.pushes)
    assert kept > 0 and n.backend.d2h_bytes_last <= 8 * (ParamLayout(CFG).num_params() // 10 + 64)
