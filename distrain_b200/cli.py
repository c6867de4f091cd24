"""Command-line interface: ``python -m distrain_b200 <command>``.

Node commands mirror the reference CLI (node/cli/src/main.rs:24-122): start, bootstrap, benchmark,
status, config, eval, gpu-stress-test, baseline, generate. Service / tooling commands: coordinator
(the HTTP coordinator, env-configured like coordinator/src/main.rs:141-188), prepare-data (the data-prep
script's random-shard mode), micro-cluster (coordinator + N CPU node processes on one host), train-box
(every GPU of this box as one node of the in-box protocol; launched with ``torch.distributed.run``).
The reference's post-training scripts (scripts/run_sft.py, run_dpo.py, run_evals.py, export_hf.py,
serve.py) are the commands sft, dpo, evals, export-hf and serve.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import signal
import subprocess
import sys
import time


def _store(path_or_url=None):
    """An object store from a directory / file:// path / http(s) endpoint, or, when none is given, the S3
    settings of the environment (R2_ENDPOINT, R2_BUCKET, R2_ACCESS_KEY_ID, R2_SECRET_ACCESS_KEY,
    R2_REGION, as the coordinator reads them)."""
    from .utils.storage import open_store
    if not path_or_url:
        from .config import CoordinatorConfig
        return open_store(CoordinatorConfig.from_env().storage)
    return open_store(path_or_url)


def _store_from_cfg(storage_cfg):
    from .utils.storage import open_store
    return open_store(storage_cfg)


def _model_cfg(preset: str, vocab=None, seq=None, theta=None):
    from .config import preset as get_preset, bench_config
    if preset in ("micro-test-bench", "micro-bench"):
        m = bench_config("micro").model
    else:
        m = get_preset(preset)
    if vocab:
        m.vocab_size = vocab
    if seq:
        m.max_seq_len = max(m.max_seq_len, seq)
    if theta:
        m.rope_theta = theta
    return m


def _infer_model_config(sd):
    """Model hyper-parameters from checkpoint shapes (reference trainer.rs:837-906). The shapes do not
    determine the head count (q_proj is [heads * head_dim, hidden] for every split), so a checkpoint
    whose hidden size, depth, FFN width and KV width match a preset takes that preset's heads (the
    vocabulary comes from the checkpoint); otherwise head_dim is the largest of 128/64/32/16 that fits."""
    from .config import ModelConfig, preset
    V, H = sd["embedding.embedding.weight"].shape
    L = 1 + max(int(k.split(".")[1]) for k in sd if k.startswith("layers."))
    qd = sd["layers.0.attention.q_proj.weight"].shape[0]
    kvd = sd["layers.0.attention.k_proj.weight"].shape[0]
    F = sd["layers.0.ffn.gate_proj.weight"].shape[0]
    bias = "layers.0.attention.q_proj.bias" in sd
    for name in ("micro", "tiny", "small", "medium", "large"):
        c = preset(name)
        d = c.hidden_dim // c.num_heads
        if (c.hidden_dim, c.num_layers, c.ffn_hidden_dim, c.num_kv_heads * d) == (H, L, F, kvd) and qd == H:
            c.vocab_size, c.qkv_bias = V, bias
            return c
    for d in (128, 64, 32, 16):
        if qd % d == 0 and kvd % d == 0 and H % d == 0 and H // d == qd // d:
            break
    return ModelConfig(hidden_dim=H, num_layers=L, num_heads=qd // d, num_kv_heads=kvd // d, ffn_hidden_dim=F,
                       vocab_size=V, qkv_bias=bias)


def _saved_node_id(cache_dir):
    """The identity this node registered with before (kept in its cache directory, reference
    main.rs:251-260), so a restarted node is the same node to the coordinator."""
    path = os.path.join(cache_dir, "node_id") if cache_dir else None
    if path and os.path.exists(path):
        with open(path) as f:
            return f.read().strip() or None
    return None


def _save_node_id(cache_dir, node_id):
    if cache_dir and node_id:
        os.makedirs(cache_dir, exist_ok=True)
        with open(os.path.join(cache_dir, "node_id"), "w") as f:
            f.write(node_id)


def _store_data_source(store, node_id: str, batch: int, seq: int, cache_dir: str):
    """The reference node's data path (node/cli/src/continuous.rs:796-826): the shards listed in the store's
    data/manifest.json, this node's share by the deterministic assignment (node id, version 0: fixed
    across checkpoints), fetched into a local cache and read sequentially. None when the store has no
    manifest."""
    from . import protocol as P
    from .config import TrainingParams
    from .utils.data import StreamingLoader
    from .utils.native import shard_assignment
    if not store.exists(P.manifest_path()):
        return None
    total = len(store.get_json(P.manifest_path())["shards"])
    idx = shard_assignment(node_id, 0, total, TrainingParams().shards_per_node(total))
    return StreamingLoader(store, cache_dir, idx, seq, batch, max_resident=4, prefetch=0).next_batch


def _data_source(args, vocab, batch, seq, seed):
    if getattr(args, "data_dir", None):
        from .utils.data import ShardLoader
        files = sorted(os.path.join(args.data_dir, f) for f in os.listdir(args.data_dir) if f.endswith(".bin"))
        loader = ShardLoader(files, seq, batch, max_resident=8)
        if getattr(args, "seek_seed", None) is not None:
            loader.seek_by_seed(args.seek_seed)
        return loader.next_batch
    from .utils.data import SyntheticTokens
    return SyntheticTokens(vocab, batch, seq, seed).next_batch


# ─────────────────────────────── commands ───────────────────────────────
def cmd_coordinator(args):
    from .config import CoordinatorConfig
    from .coordinator.service import CoordinatorService
    cfg = CoordinatorConfig.from_env()
    if args.port is not None:
        cfg.port = args.port
    store = _store(args.store) if args.store else _store_from_cfg(cfg.storage)
    store.ensure_bucket()
    svc = CoordinatorService(cfg, store, merge_device=args.merge_device)
    port = svc.start(host=args.host or cfg.host)
    print(json.dumps({"event": "coordinator_started", "port": port}), flush=True)
    stop = []
    signal.signal(signal.SIGTERM, lambda *a: stop.append(1))
    try:
        while not stop:
            time.sleep(0.5)
    except KeyboardInterrupt:
        pass
    svc.stop()


def cmd_bootstrap(args):
    from .coordinator.service import bootstrap
    from . import protocol as P
    store = _store(args.store)
    if args.if_absent and store.exists(P.checkpoint_path(0)):
        print(json.dumps({"event": "bootstrap_skipped", "reason": "checkpoint v0 exists"}))
        return
    init = None
    if args.from_hf:
        from .utils.hf_export import from_hf
        init, m = from_hf(args.from_hf)
    else:
        m = _model_cfg(args.preset, args.vocab, args.seq_len, args.rope_theta)
    L, _ = bootstrap(store, m, seed=args.seed, init_state=init)
    print(json.dumps({"event": "bootstrapped", "version": 0, "params": L.num_params(), "model": m.to_dict()}))


def _apply_node_config(args):
    """Fill the start command's unset options from a node.toml (the reference's NodeConfig,
    core/shared/src/config.rs:81-143): coordinator_url, [storage], gpu_device, force_batch_size /
    batch_size, seq_len, force_cpu, min_inner_steps (steps per push). Flags win over the file; without a
    file the storage comes from the R2_* environment."""
    from .config import CoordinatorConfig, NodeConfig
    nc = NodeConfig.load_toml(args.config) if args.config else None
    args.max_memory_fraction = nc.max_memory_fraction if nc is not None else NodeConfig().max_memory_fraction
    if nc is None:
        args.storage_cfg = CoordinatorConfig.from_env().storage
    else:
        args.storage_cfg = nc.storage
        if not args.coordinator_url:
            args.coordinator_url = nc.coordinator_url
        if args.device is None and not args.cpu:
            if nc.force_cpu:
                args.cpu = True
            elif nc.gpu_device >= 0:
                args.device = f"cuda:{nc.gpu_device}"
        if args.batch_size is None:
            args.batch_size = nc.force_batch_size or nc.batch_size
        if args.seq_len is None:
            args.seq_len = nc.seq_len
        if args.h_mini is None and nc.min_inner_steps:
            args.h_mini = nc.min_inner_steps
        if args.h_mini_bounds is None:
            args.h_mini_bounds = (nc.min_inner_steps, nc.max_inner_steps)
        if getattr(args, "cache_dir", None) is None and nc.cache_dir:
            args.cache_dir = os.path.expanduser(nc.cache_dir)
    if not args.coordinator_url:
        raise SystemExit("start: --coordinator-url or a --config with coordinator_url is required")
    if args.batch_size is None and args.cpu:
        args.batch_size = 4  # on a GPU an unset batch size is calibrated against the device (cmd_start)
    args.seq_len = args.seq_len or 512
    args.h_mini = args.h_mini or 50


def cmd_start(args):
    from .config import CompressionConfig, OptimConfig
    from .parallel.http_node import HttpNode
    from .utils.checkpoint import load_safetensors_bytes
    from .coordinator.client import CoordinatorClient
    from . import protocol as P
    _apply_node_config(args)
    store = _store(args.store) if args.store else _store_from_cfg(args.storage_cfg)
    cl = CoordinatorClient(args.coordinator_url)
    v = cl.get_latest_checkpoint().version
    m = _infer_model_config(load_safetensors_bytes(store.get(P.checkpoint_path(v))))
    if args.rope_theta:
        m.rope_theta = args.rope_theta
    m.max_seq_len = max(m.max_seq_len, args.seq_len)
    device = "cpu" if args.cpu else (args.device or "cuda:0")
    if args.batch_size is None:
        args.batch_size = _calibrated_batch(store.get(P.checkpoint_path(v)), args.seq_len, device)

    def make(batch, node_id):
        node = HttpNode(args.coordinator_url, store, m, batch, args.seq_len, h_mini=args.h_mini,
                        optim=OptimConfig(lr=args.lr), compression=CompressionConfig(top_k_fraction=args.top_k,
                                                                                     quantize_int8=not args.no_int8),
                        device=device, node_id=node_id, data=None, poll_secs=args.poll_secs,
                        bandwidth_adaptive=args.bandwidth_adaptive, resume_path=args.resume_file,
                        resume_every=args.resume_every, max_memory_fraction=args.max_memory_fraction,
                        h_mini_bounds=args.h_mini_bounds, ckpt_cache_dir=args.cache_dir)
        node.register(gpu_model="cpu" if device == "cpu" else "B200")
        _save_node_id(args.cache_dir, node.node_id)
        # data: local shards (--data-dir), else this node's assigned shards from the store, else synthetic
        node.data = None if args.data_dir or args.synthetic_data else _store_data_source(
            store, node.node_id, batch, args.seq_len, args.cache_dir or os.path.join(
                os.path.expanduser("~"), ".distrain", "cache", node.node_id))
        if node.data is None:
            node.data = _data_source(args, m.vocab_size, batch, args.seq_len, args.seed)
        return node
    node, log = run_with_oom_halving(make, args.batch_size, args.steps, args.node_id or _saved_node_id(args.cache_dir))
    out = {"event": "node_done", "node_id": node.node_id, "steps": len(log), "version": node.version,
           "resumed": node.resumed, "global_step": node.global_step,
           "first_loss": log[0]["loss"] if log else None, "last_loss": log[-1]["loss"] if log else None,
           "pushes": len(node.pushes), "accepted": sum(p["accepted"] for p in node.pushes), "errors": node.errors}
    if args.metrics_out:
        with open(args.metrics_out, "w") as f:
            for r in log:
                f.write(json.dumps(r) + "\n")
    print(json.dumps(out), flush=True)


def run_with_oom_halving(make, batch: int, steps: int, node_id=None):
    """Build a node at `batch` and train; on a device out-of-memory error rebuild it at half the batch under
    the same identity (its resume file carries it on), down to batch 1, after which the error stands
    (reference main.rs:790-827, continuous.rs:919-934). Returns (node, log)."""
    import torch
    while True:
        node = None
        try:
            node = make(batch, node_id)
            return node, node.run(steps)
        except torch.cuda.OutOfMemoryError:
            if node is not None:
                node_id = node.node_id
            if batch <= 1:
                raise
            batch //= 2
            if torch.cuda.is_available():
                torch.cuda.empty_cache()
            print(json.dumps({"event": "oom_halved_batch", "batch_size": batch}), flush=True)


def apply_run_overrides(run, args):
    """Command-line overrides of a RunConfig (train-box); unset flags keep the preset's values."""
    for flag, field_name in (("push_every", "push_every"), ("tp", "tp"), ("checkpoint_store", "checkpoint_store"),
                             ("checkpoint_every", "checkpoint_every"), ("keep_versions", "keep_versions"),
                             ("metrics_port", "metrics_port"), ("watchdog_secs", "watchdog_step_secs"),
                             ("swap_mode", "swap_mode"), ("ef_on_swap", "ef_on_swap"), ("seed", "seed"),
                             ("payload_slots", "payload_slots")):
        v = getattr(args, flag, None)
        if v is not None:
            setattr(run, field_name, v)
    for flag, field_name in (("resume", "resume"), ("loss_based_lr", "loss_based_lr"),
                             ("bandwidth_adaptive", "bandwidth_adaptive"),
                             ("reset_optimizer", "reset_optimizer_on_swap"),
                             ("activation_checkpointing", "activation_checkpointing")):
        if getattr(args, flag, False):
            setattr(run, field_name, True)
    if getattr(args, "top_k", None) is not None:
        run.compression.top_k_fraction = args.top_k
    if getattr(args, "no_int8", False):
        run.compression.quantize_int8 = False
    if getattr(args, "lr", None) is not None:
        run.optim.lr = args.lr
    if getattr(args, "batch_size", None) is not None:
        run.micro_batch = args.batch_size
    if getattr(args, "grad_accum", None) is not None:
        run.grad_accum_steps = max(int(args.grad_accum), 1)
    if getattr(args, "merge_sms", None) is not None:
        run.merge_sms = max(int(args.merge_sms), 0)
    if getattr(args, "seq_len", None) is not None:
        run.seq_len = args.seq_len
        run.model.max_seq_len = max(run.model.max_seq_len, args.seq_len)
    return run


def cmd_train_box(args):
    """In-box training job: one node per GPU process (rank), the compressed protocol over NVLink between
    them, batches from local token shards (each node its deterministic share) or synthetic tokens."""
    import torch
    import torch.distributed as dist
    from .config import bench_config
    from .parallel.launch import init_box, box_node, node_batches, node_layout, restore_data_state, save_data_state
    br = init_box(args.pg_timeout)
    run = apply_run_overrides(bench_config(args.preset), args)
    node, node_rank, n_nodes = box_node(run, br, enable_push=not args.no_push, tp_mode=args.tp_mode, sync=args.sync)
    source, desc = node_batches(run, node_rank, n_nodes, args.data_dir, args.shards_fraction, run.seed)
    # with a checkpoint store every node also keeps its data position there (one writer per node)
    dstore = _store(run.checkpoint_store) if run.checkpoint_store else None
    data_resumed = bool(dstore is not None and run.resume and restore_data_state(dstore, node_rank, source))
    writes_data = dstore is not None and br.rank % node_layout(br.world, run.tp)[0] == 0
    out = open(args.output, "w") if (args.output and br.rank == 0) else None

    def emit(rec):
        if br.rank == 0:
            print(json.dumps(rec), flush=True)
            if out:
                out.write(json.dumps(rec) + "\n")
                out.flush()
    emit({"event": "train_box_start", "preset": run.name, "nodes": n_nodes, "ranks": br.world, "tp": run.tp,
          "micro_batch": run.micro_batch, "grad_accum_steps": run.grad_accum_steps, "seq_len": run.seq_len,
          "push_every": run.push_every, "data": desc,
          "resumed_version": getattr(node.sync, "resumed_version", 0), "data_resumed": data_resumed})
    done = 0
    tokens_per_step = run.grad_accum_steps * run.micro_batch * (run.seq_len - 1) * n_nodes
    while done < args.steps:
        k = min(args.log_every, args.steps - done)
        t0 = time.time()
        losses = node.train_stream(source, k)
        dt = time.time() - t0
        done += k
        if writes_data:
            save_data_state(dstore, node_rank, source)
        emit({"event": "train", "step": done, "loss": sum(losses) / len(losses), "last_loss": losses[-1],
              "tokens_per_sec": tokens_per_step * k / dt, "version": getattr(node.sync, "version", 0)})
        if getattr(node, "hung", None):
            emit({"event": "watchdog", "detail": str(node.hung)})
            break
    node.close()
    if br.world > 1:
        dist.barrier()
    emit({"event": "train_box_done", "steps": done, "version": getattr(node.sync, "version", 0),
          "merges": len(getattr(node.sync, "merges", []) or [])})
    if out:
        out.close()
    if br.world > 1:
        dist.destroy_process_group()


def cmd_status(args):
    from .coordinator.client import CoordinatorClient
    print(json.dumps(CoordinatorClient(args.coordinator_url).get_status().to_dict(), indent=2))


def cmd_config(args):
    from .config import TrainingParams
    out = {"local_training_params": TrainingParams().to_dict()}
    if args.coordinator_url:
        from .coordinator.client import CoordinatorClient
        out["coordinator"] = CoordinatorClient(args.coordinator_url).get_config()
    print(json.dumps(out, indent=2))


def _eval_loss(sd, cfg, batches, device):
    """Mean next-token loss over ``batches`` ([B, S] token ids each): on a GPU through the CUDA engine's
    forward-only pass, else through the fp32 formulation."""
    import torch
    from .models import oracle
    if torch.device(device).type == "cuda" and batches:
        from .models.engine import TrainEngine
        from .models.params import ParamLayout
        L = ParamLayout(cfg)
        flat = torch.zeros(L.total)
        L.load_state_dict(flat, {k: v.detach().float().cpu() for k, v in sd.items()})
        B, S = batches[0].shape
        eng = TrainEngine(cfg, B, S, device=device, flat_init=flat, inference=True)
        tot = 0.0
        for b in batches:
            eng.set_tokens(b.to(device).int())
            tot += float(eng.forward_loss(0).double().mean())
        return tot / len(batches)
    p = {k: v.to(device) for k, v in sd.items()}
    tot = 0.0
    with torch.no_grad():
        for b in batches:
            tot += float(oracle.lm_loss(p, cfg, b.to(device).long()).item())
    return tot / max(len(batches), 1)


def cmd_eval(args):
    import torch
    from .utils.checkpoint import load_safetensors
    res = []
    for ck in args.checkpoints:
        sd = load_safetensors(ck)
        cfg = _infer_model_config(sd)
        if args.rope_theta:
            cfg.rope_theta = args.rope_theta
        cfg.max_seq_len = max(cfg.max_seq_len, args.seq_len)
        src = _data_source(args, cfg.vocab_size, args.batch_size, args.seq_len, args.seed)
        batches = [src() for _ in range(args.batches)]
        dev = args.device or ("cuda:0" if torch.cuda.is_available() else "cpu")
        res.append({"checkpoint": ck, "loss": _eval_loss(sd, cfg, batches, dev), "batches": args.batches})
    print(json.dumps(res, indent=2))


def cmd_baseline(args):
    """Single-device baseline (no coordinator, no compression), cosine LR with warmup, JSONL per step
    (reference main.rs:1110-1216)."""
    import torch
    from .config import cosine_lr, OptimConfig
    from .utils.checkpoint import load_safetensors
    sd = load_safetensors(args.checkpoint)
    cfg = _infer_model_config(sd)
    if args.rope_theta:
        cfg.rope_theta = args.rope_theta
    cfg.max_seq_len = max(cfg.max_seq_len, args.seq_len)
    src = _data_source(args, cfg.vocab_size, args.batch_size, args.seq_len, args.seed)
    warm = int(args.steps * 0.2)
    if args.cpu:
        from .parallel.http_node import CpuBackend
        be = CpuBackend(cfg, OptimConfig(lr=args.lr_max))
        be.load(sd)
        step = lambda toks, lr: be.step(toks, lr)
    else:
        from .models.engine import TrainEngine
        from .models.params import ParamLayout
        L = ParamLayout(cfg)
        flat = torch.zeros(L.total)
        L.load_state_dict(flat, sd)
        eng = TrainEngine(cfg, args.batch_size, args.seq_len, optim=OptimConfig(lr=args.lr_max),
                          device=args.device or "cuda:0", flat_init=flat)

        def step(toks, lr):
            eng.set_lr(lr)
            eng.set_tokens(toks.to(eng.device))
            eng.step()
            return float(eng.loss[0].item())
    with open(args.output, "w") as f:
        for s in range(args.steps):
            lr = cosine_lr(s, warm, args.steps, args.lr_max, args.lr_max * 0.1)
            loss = step(src(), lr)
            f.write(json.dumps({"step": s + 1, "loss": loss, "lr": lr,
                                "tokens": (s + 1) * args.batch_size * args.seq_len}) + "\n")
    print(json.dumps({"event": "baseline_done", "steps": args.steps, "output": args.output}))


def torch_device_is_cuda(device) -> bool:
    return bool(device) and str(device).startswith("cuda")


def cmd_generate(args):
    """Greedy / temperature sampling by full re-forward (the reference has no KV cache, main.rs:1416-1548)."""
    from .serve import load_model, sample
    sd, cfg = load_model(args.checkpoint, getattr(args, "device", None) or "cpu", args.rope_theta,
                         min_len=args.max_tokens + 64)
    ids = [int(x) for x in args.prompt_ids.split(",")] if args.prompt_ids else [1]
    tok = None
    if args.tokenizer == "bytes":  # the UTF-8 byte tokenizer of the post-training commands
        from .alignment import ByteTokenizer
        tok = ByteTokenizer()
        ids = tok.encode(args.prompt)
    elif args.tokenizer:
        from tokenizers import Tokenizer
        tok = Tokenizer.from_file(args.tokenizer)
        ids = tok.encode(args.prompt).ids
    lm = None
    if torch_device_is_cuda(getattr(args, "device", None)):
        from .serve import EngineLM
        lm = EngineLM(sd, cfg, args.device, window=len(ids) + args.max_tokens)
    new, _ = sample(sd, cfg, ids, args.max_tokens, args.temperature, args.seed, lm=lm)
    ids = ids + new
    print(json.dumps({"ids": ids, "text": tok.decode(ids) if tok else None}))


def cmd_serve(args):
    """OpenAI-style completion server for one checkpoint (the reference's scripts/serve.py:16,32-37)."""
    import time as _time
    from .serve import CompletionServer
    srv = CompletionServer(args.checkpoint, args.device or "cpu", args.tokenizer, args.rope_theta,
                           model_name=args.model_name, max_tokens_cap=args.max_tokens_cap, template=args.template)
    port = srv.start(args.host, args.port)
    print(json.dumps({"serving": args.checkpoint, "port": port, "model": srv.model}), flush=True)
    try:
        while True:
            _time.sleep(3600)
    except KeyboardInterrupt:
        srv.stop()


def _posttrain_model(args, checkpoint):
    """(ModelConfig, flat fp32 weights) of a post-training run: a checkpoint, or a random model of
    ``--model-size``."""
    import torch
    from .models.params import ParamLayout, init_flat
    if checkpoint:
        from .utils.checkpoint import load_safetensors
        sd = load_safetensors(checkpoint)
        cfg = _infer_model_config(sd)
        L = ParamLayout(cfg)
        flat = torch.zeros(L.total)
        L.load_state_dict(flat, sd)
    else:
        cfg = _model_cfg(args.model_size, vocab=args.vocab)
        flat = init_flat(ParamLayout(cfg), seed=args.seed)
    if args.rope_theta:
        cfg.rope_theta = args.rope_theta
    cfg.max_seq_len = max(cfg.max_seq_len, args.max_seq_len)
    return cfg, flat


def _posttrain_tokenizer(args, cfg):
    from .alignment import ByteTokenizer, FileTokenizer
    tok = FileTokenizer(args.tokenizer) if args.tokenizer else ByteTokenizer()
    if tok.vocab_size > cfg.vocab_size:
        raise SystemExit(f"tokenizer vocabulary {tok.vocab_size} > model vocabulary {cfg.vocab_size}")
    return tok


def _posttrain_done(event, m, keys):
    print(json.dumps({"event": event, **{k: m[k] for k in keys}}))


def cmd_sft(args):
    """Supervised fine-tuning on chat data, loss on the assistant turns (the reference's scripts/run_sft.py)."""
    from .alignment import SFTConfig, SFTTrainer, load_chat_jsonl, synthetic_conversations, tokenize_conversation
    cfg, flat = _posttrain_model(args, args.base_model)
    tok = _posttrain_tokenizer(args, cfg)
    if args.synthetic:
        convs = synthetic_conversations(args.max_examples or 100)
    elif args.datasets:
        convs = load_chat_jsonl([d.strip() for d in args.datasets.split(",")], args.max_examples)
    else:
        raise SystemExit("sft: give --datasets (JSONL files) or --synthetic")
    examples = [tokenize_conversation(c, tok, args.template, args.max_seq_len) for c in convs]
    c = SFTConfig(learning_rate=args.lr, num_epochs=args.epochs, batch_size=args.batch_size,
                  gradient_accumulation_steps=args.grad_accum, max_seq_len=args.max_seq_len,
                  save_every_n_steps=args.save_every, log_every_n_steps=args.log_every, output_dir=args.output,
                  seed=args.seed, use_lora=args.use_lora, lora_rank=args.lora_rank, lora_alpha=args.lora_alpha)
    m = SFTTrainer(cfg, flat, examples, c, pad_id=tok.pad_id, device=args.device).train()
    _posttrain_done("sft_done", m, ("steps", "examples", "response_tokens", "first_loss", "final_loss",
                                    "tokens_per_sec", "checkpoint"))


def cmd_dpo(args):
    """Direct preference optimisation against the frozen starting model (the reference's scripts/run_dpo.py)."""
    from .alignment import DPOConfig, DPOTrainer, load_preference_jsonl, synthetic_preferences
    cfg, flat = _posttrain_model(args, args.sft_model)
    pad_id = 0
    if args.synthetic:  # token ids 1..48, no tokenizer
        pairs = synthetic_preferences(args.max_examples or 50)
    elif args.datasets:
        tok = _posttrain_tokenizer(args, cfg)
        pad_id = tok.pad_id
        pairs = load_preference_jsonl([d.strip() for d in args.datasets.split(",")], tok, args.template,
                                      args.max_examples)
    else:
        raise SystemExit("dpo: give --datasets (JSONL files) or --synthetic")
    c = DPOConfig(beta=args.beta, learning_rate=args.lr, num_epochs=args.epochs, batch_size=args.batch_size,
                  gradient_accumulation_steps=args.grad_accum, max_seq_len=args.max_seq_len,
                  save_every_n_steps=args.save_every, log_every_n_steps=args.log_every, output_dir=args.output,
                  seed=args.seed, use_lora=args.use_lora, lora_rank=args.lora_rank, lora_alpha=args.lora_alpha)
    m = DPOTrainer(cfg, flat, pairs, c, pad_id=pad_id, device=args.device).train()
    _posttrain_done("dpo_done", m, ("steps", "pairs", "first_loss", "final_loss", "final_reward_accuracy",
                                    "pairs_per_sec", "checkpoint"))


def cmd_evals(args):
    """Multiple-choice benchmark scores of checkpoints from local task files (the reference's
    scripts/run_evals.py)."""
    from .evaluation import (FULL_TASKS, QUICK_TASKS, evaluate_checkpoint, find_checkpoint, save_result,
                             summary_table)
    tasks = QUICK_TASKS if args.quick else ([t.strip() for t in args.tasks.split(",")] if args.tasks else FULL_TASKS)
    if args.checkpoint:
        todo = [(args.checkpoint, None)]
    else:
        if not args.versions:
            raise SystemExit("evals: --versions is required with --checkpoint-dir")
        todo = []
        for v in (int(x) for x in args.versions.split(",")):
            try:
                todo.append((find_checkpoint(args.checkpoint_dir, v), v))
            except FileNotFoundError as e:
                print(f"warning: {e}", file=sys.stderr)
    results = []
    for ck, v in todo:
        r = evaluate_checkpoint(ck, tasks, args.task_dir, args.model_size, args.device, args.batch_size,
                                args.seq_len, args.limit, args.tokenizer, v, args.vocab, args.seed)
        path = save_result(r, args.output_dir)
        results.append(r)
        print(summary_table(r), file=sys.stderr)
        print(json.dumps({"event": "evals", "checkpoint": ck, "version": v, "results": r["results"],
                          "output": path}))
    if args.plot and len(results) > 1:
        try:
            import matplotlib
            matplotlib.use("Agg")
            import matplotlib.pyplot as plt
        except ImportError:
            print("warning: matplotlib is not installed; no plot", file=sys.stderr)
            return
        fig, ax = plt.subplots(figsize=(10, 6))
        for task in tasks:
            pts = sorted((r["version"], x["acc"]) for r in results for x in r["results"] if x["task"] == task)
            ax.plot([p[0] for p in pts], [p[1] for p in pts], marker="o", label=task)
        ax.set_xlabel("checkpoint version")
        ax.set_ylabel("acc")
        ax.legend()
        fig.savefig(os.path.join(args.output_dir, "eval_curves.png"), dpi=150)


def cmd_benchmark(args):
    """Measure this device's training step time and the largest batch that fits (calibration)."""
    import torch
    from .config import bench_config
    from .models.engine import TrainEngine
    run = bench_config(args.preset)
    eng = TrainEngine(run.model, args.batch_size or run.micro_batch, args.seq_len or run.seq_len,
                      device=args.device or "cuda:0")
    toks = torch.randint(0, run.model.vocab_size, (eng.B, eng.S), dtype=torch.int32, device=eng.device)
    eng.set_tokens(toks)
    eng.capture()
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        eng.step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    free, total = torch.cuda.mem_get_info()
    print(json.dumps({"preset": args.preset, "batch": eng.B, "seq_len": eng.S, "ms_per_step": round(ms, 3),
                      "tokens_per_sec": round(eng.B * eng.S / ms * 1e3, 1),
                      "mem_used_gb": round((total - free) / 2 ** 30, 2), "mem_total_gb": round(total / 2 ** 30, 2)}))


def cmd_gpu_stress_test(args):
    """Child-process probe: one step at (batch, seq) from a checkpoint; exit 0 if it fits (trainer.rs:776-827)."""
    import torch
    from .utils.checkpoint import load_safetensors
    from .models.engine import TrainEngine
    from .models.params import ParamLayout
    sd = load_safetensors(args.checkpoint)
    cfg = _infer_model_config(sd)
    cfg.max_seq_len = max(cfg.max_seq_len, args.seq_len)
    try:
        L = ParamLayout(cfg)
        flat = torch.zeros(L.total)
        L.load_state_dict(flat, sd)
        eng = TrainEngine(cfg, args.batch_size, args.seq_len, device=args.device or "cuda:0", flat_init=flat)
        eng.set_tokens(torch.randint(0, cfg.vocab_size, (eng.B, eng.S), dtype=torch.int32, device=eng.device))
        eng.step_kernels()
        torch.cuda.synchronize()
        ok = math.isfinite(eng.loss[0].item())
    except torch.cuda.OutOfMemoryError:
        ok = False
    print(json.dumps({"batch_size": args.batch_size, "seq_len": args.seq_len, "fits": ok}))
    sys.exit(0 if ok else 3)


def _calibrated_batch(ckpt_bytes: bytes, seq_len: int, device: str) -> int:
    """The largest batch that trains on this device (no batch size forced by flag or config, as the
    reference node calibrates before it registers, main.rs:600-618)."""
    import tempfile
    with tempfile.NamedTemporaryFile(suffix=".safetensors") as f:
        f.write(ckpt_bytes)
        f.flush()
        best = calibrate_batch_size(f.name, seq_len, device=device)
    if best < 1:
        raise SystemExit(f"start: not even batch 1 at seq_len {seq_len} fits on {device}")
    print(json.dumps({"event": "batch_calibrated", "batch_size": best, "seq_len": seq_len}), flush=True)
    return best


def calibrate_batch_size(checkpoint: str, seq_len: int, lo: int = 1, hi: int = 256, device="cuda:0",
                         probe_timeout: float = 300.0) -> int:
    """Binary search of the largest batch that fits, each probe in a child process so an out-of-memory
    failure cannot take down the caller (reference trainer.rs:733-834)."""
    best = 0
    while lo <= hi:
        mid = (lo + hi) // 2
        try:  # a probe that does not finish in time counts as not fitting (reference trainer.rs:322-359)
            r = subprocess.run([sys.executable, "-m", "distrain_b200", "gpu-stress-test", checkpoint, "--batch-size",
                                str(mid), "--seq-len", str(seq_len), "--device", device], capture_output=True,
                               timeout=probe_timeout)
            ok = r.returncode == 0
        except subprocess.TimeoutExpired:
            ok = False
        if ok:
            best, lo = mid, mid + 1
        else:
            hi = mid - 1
    return best


def load_safetensors_bytes_from(store, version: int):
    from . import protocol as P
    from .utils.checkpoint import load_safetensors_bytes
    return load_safetensors_bytes(store.get(P.checkpoint_path(version)))


def cmd_export_hf(args):
    """Checkpoint -> Hugging Face Qwen2ForCausalLM directory (config.json + model.safetensors)."""
    from .utils.checkpoint import load_safetensors
    from .utils.hf_export import export_hf
    if args.store:  # a stored version, whole or tensor-parallel shards (model-tp{t}of{T}), gathered
        from .parallel.inbox_ckpt import gather_checkpoint, latest_version
        st = _store(args.store)
        v = args.version if args.version is not None else latest_version(st, args.tp)
        if v is None:
            raise SystemExit(f"export-hf: no stored checkpoint for {args.tp} shard(s) in {args.store}")
        sd = gather_checkpoint(st, v, args.tp) if args.tp > 1 else load_safetensors_bytes_from(st, v)
    else:
        sd = load_safetensors(args.checkpoint)
    cfg = _infer_model_config(sd)
    if args.rope_theta:
        cfg.rope_theta = args.rope_theta
    if args.max_seq_len:
        cfg.max_seq_len = args.max_seq_len
    export_hf(sd, cfg, args.output_dir)
    print(json.dumps({"event": "exported_hf", "output_dir": args.output_dir, "architecture": "Qwen2ForCausalLM",
                      "model": cfg.to_dict()}))


def cmd_prepare_data(args):
    from .utils.data import prepare_random_shards, iter_text_documents, tokenize_to_shards
    if args.input:
        if not args.tokenizer:
            raise SystemExit("prepare-data --input needs --tokenizer (a tokenizers JSON file)")
        m = tokenize_to_shards(iter_text_documents(args.input, args.text_column, args.max_samples), args.output_dir,
                               args.tokenizer, args.vocab, args.tokens_per_shard)
    else:
        m = prepare_random_shards(args.output_dir, args.num_shards, args.tokens_per_shard, args.vocab, args.seed)
    if args.upload_store:
        st = _store(args.upload_store)
        for f in os.listdir(args.output_dir):
            key = "data/manifest.json" if f == "manifest.json" else f"data/{f}"
            st.upload_from_file(os.path.join(args.output_dir, f), key)
    print(json.dumps({"event": "prepared", "num_shards": m["num_shards"], "total_tokens": m["total_tokens"]}))


def cmd_micro_cluster(args):
    """Coordinator + N CPU node processes on the micro-test workload (vocab 32768, seq 128, batch 4,
    theta 1e4, push every 20 steps, top-k 10% + INT8)."""
    import tempfile
    root = args.store or tempfile.mkdtemp(prefix="distrain-micro-")
    env = dict(os.environ, PORT=str(args.port), MIN_CONTRIBUTIONS="0", OUTER_LR="1.0", OUTER_MOMENTUM="0.0")
    py = [sys.executable, "-m", "distrain_b200"]
    subprocess.run(py + ["bootstrap", "--preset", "micro-bench", "--store", root, "--seed", "0"], check=True, env=env)
    coord = subprocess.Popen(py + ["coordinator", "--store", root, "--host", "127.0.0.1"], env=env,
                             stdout=subprocess.PIPE, text=True)
    coord.stdout.readline()
    url = f"http://127.0.0.1:{args.port}"
    nodes = [subprocess.Popen(py + ["start", "--coordinator-url", url, "--store", root, "--cpu", "--steps",
                                    str(args.steps), "--batch-size", "4", "--seq-len", "128", "--h-mini", "20",
                                    "--rope-theta", "10000", "--node-id", f"micro-{i}", "--seed", str(100 + i),
                                    "--poll-secs", "1"], env=env, stdout=subprocess.PIPE, text=True)
             for i in range(args.nodes)]
    outs = [json.loads(n.communicate()[0].strip().splitlines()[-1]) for n in nodes]
    coord.send_signal(signal.SIGTERM)
    coord.wait(timeout=60)
    print(json.dumps({"event": "micro_cluster_done", "store": root, "nodes": outs}))


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="distrain_b200")
    sp = ap.add_subparsers(dest="cmd", required=True)

    p = sp.add_parser("coordinator", help="run the coordinator HTTP service")
    p.add_argument("--store", help="object store: directory / file:// path, or http(s):// S3 endpoint "
                                    "(default: the R2_* environment)")
    p.add_argument("--host")
    p.add_argument("--port", type=int)
    p.add_argument("--merge-device", default="cpu")
    p.set_defaults(fn=cmd_coordinator)

    p = sp.add_parser("bootstrap", help="create and store checkpoint v0")
    p.add_argument("--store", help="default: the R2_* environment")
    p.add_argument("--if-absent", action="store_true", help="do nothing when checkpoint v0 already exists")
    p.add_argument("--from-hf", help="start from a pretrained Hugging Face Qwen2-layout directory")
    p.add_argument("--preset", default="tiny")
    p.add_argument("--vocab", type=int)
    p.add_argument("--seq-len", type=int)
    p.add_argument("--rope-theta", type=float)
    p.add_argument("--seed", type=int, default=0)
    p.set_defaults(fn=cmd_bootstrap)

    p = sp.add_parser("start", help="run a training node against a coordinator")
    p.add_argument("--config", help="node.toml (coordinator_url, [storage], gpu_device, batch size, seq_len)")
    p.add_argument("--coordinator-url")
    p.add_argument("--store", help="default: the config's [storage], else the R2_* environment")
    p.add_argument("--cpu", action="store_true")
    p.add_argument("--device")
    p.add_argument("--node-id")
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--batch-size", type=int, help="default: the config's, else 4")
    p.add_argument("--seq-len", type=int, help="default: the config's, else 512")
    p.add_argument("--h-mini", type=int, help="steps per push (default: the config's min_inner_steps, else 50)")
    p.add_argument("--lr", type=float, default=3e-4)
    p.add_argument("--top-k", type=float, default=0.1)
    p.add_argument("--no-int8", action="store_true")
    p.add_argument("--bandwidth-adaptive", action="store_true")
    p.add_argument("--data-dir")
    p.add_argument("--seek-seed", type=int)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--rope-theta", type=float)
    p.add_argument("--poll-secs", type=float, default=5.0)
    p.add_argument("--metrics-out")
    p.add_argument("--cache-dir", help="shard cache for data streamed from the store (default ~/.distrain/cache/<id>)")
    p.add_argument("--auto-h-mini", dest="h_mini_bounds", type=lambda v: tuple(int(x) for x in v.split(",")),
                   help="MIN,MAX: retune the steps per push at each checkpoint from the upload bandwidth "
                        "(default with --config: its min/max_inner_steps)")
    p.add_argument("--synthetic-data", action="store_true", help="uniform random tokens even if the store has data")
    p.add_argument("--resume-file", help="node-local resume file: written at round boundaries, read at start "
                                         "(same checkpoint: weights, AdamW and error feedback continue; newer: "
                                         "identity, step count and data position continue)")
    p.add_argument("--resume-every", type=int, default=1, help="write the resume file every N full-round pushes")
    p.set_defaults(fn=cmd_start)

    p = sp.add_parser("status", help="coordinator training status")
    p.add_argument("--coordinator-url", required=True)
    p.set_defaults(fn=cmd_status)

    p = sp.add_parser("config", help="effective training parameters")
    p.add_argument("--coordinator-url")
    p.set_defaults(fn=cmd_config)

    p = sp.add_parser("eval", help="loss of checkpoint(s) on data without training")
    p.add_argument("checkpoints", nargs="+")
    p.add_argument("--batches", type=int, default=50)
    p.add_argument("--batch-size", type=int, default=4)
    p.add_argument("--seq-len", type=int, default=512)
    p.add_argument("--data-dir")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device")
    p.add_argument("--rope-theta", type=float)
    p.set_defaults(fn=cmd_eval)

    p = sp.add_parser("baseline", help="single-device baseline training, JSONL metrics")
    p.add_argument("checkpoint")
    p.add_argument("--data-dir")
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--output", default="baseline.jsonl")
    p.add_argument("--cpu", action="store_true")
    p.add_argument("--device")
    p.add_argument("--batch-size", type=int, default=4)
    p.add_argument("--seq-len", type=int, default=512)
    p.add_argument("--lr-max", type=float, default=3e-4)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--rope-theta", type=float)
    p.set_defaults(fn=cmd_baseline)

    p = sp.add_parser("generate", help="sample tokens from a checkpoint")
    p.add_argument("checkpoint")
    p.add_argument("--prompt", default="The")
    p.add_argument("--prompt-ids")
    p.add_argument("--tokenizer", help="tokenizer JSON, or 'bytes' (UTF-8 bytes)")
    p.add_argument("--max-tokens", type=int, default=32)
    p.add_argument("--temperature", type=float, default=0.0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--rope-theta", type=float)
    p.add_argument("--device", help="torch device for the forward (default cpu)")
    p.set_defaults(fn=cmd_generate)

    p = sp.add_parser("serve", help="OpenAI-style server for a checkpoint (/v1/completions, /v1/chat/completions)")
    p.add_argument("checkpoint", help="a safetensors file, or a directory holding model.safetensors")
    p.add_argument("--tokenizer", help="tokenizer JSON, or 'bytes' (UTF-8 bytes, as the post-training commands "
                                       "use without one); token-id prompts work without a tokenizer")
    p.add_argument("--model-name", help="the model id the API reports (default: the file name)")
    p.add_argument("--template", default="chatml", choices=["chatml", "llama", "zephyr"],
                   help="chat template of /v1/chat/completions")
    p.add_argument("--host", default="0.0.0.0")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--device", help="torch device for the forward (default cpu)")
    p.add_argument("--max-tokens-cap", type=int, default=1024)
    p.add_argument("--rope-theta", type=float)
    p.set_defaults(fn=cmd_serve)

    p = sp.add_parser("evals", help="multiple-choice benchmark scores of checkpoints (local JSONL task files)")
    g = p.add_mutually_exclusive_group(required=True)
    g.add_argument("--checkpoint", help="a safetensors file, or 'random' for an untrained model")
    g.add_argument("--checkpoint-dir", help="directory of versioned checkpoints (with --versions)")
    p.add_argument("--versions", help="comma-separated versions under --checkpoint-dir")
    p.add_argument("--tasks", help="comma-separated task names (default: mmlu, hellaswag, arc_challenge, arc_easy)")
    p.add_argument("--quick", action="store_true", help="hellaswag only")
    p.add_argument("--task-dir", default="eval_data", help="directory holding <task>.jsonl files")
    p.add_argument("--model-size", default="125m", help="preset of the random model")
    p.add_argument("--vocab", type=int, help="vocabulary of the random model")
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--batch-size", type=int, default=8)
    p.add_argument("--seq-len", type=int, default=512, help="scoring window (longer inputs lose their left end)")
    p.add_argument("--limit", type=int, help="at most this many examples per task")
    p.add_argument("--tokenizer", help="tokenizer JSON; default: UTF-8 bytes")
    p.add_argument("--output-dir", default="eval_results")
    p.add_argument("--plot", action="store_true", help="accuracy curves over versions (needs matplotlib)")
    p.add_argument("--seed", type=int, default=0)
    p.set_defaults(fn=cmd_evals)

    for name, fn in (("sft", cmd_sft), ("dpo", cmd_dpo)):
        sft = name == "sft"
        p = sp.add_parser(name, help="supervised fine-tuning on chat data (loss on assistant turns)" if sft
                          else "direct preference optimisation against the frozen starting model")
        if sft:
            p.add_argument("--base-model", help="starting checkpoint (safetensors); default: a random model")
        else:
            p.add_argument("--sft-model", help="starting checkpoint (safetensors); default: a random model")
        p.add_argument("--model-size", default="125m", help="preset of the random model (125m, 1b, 7b, 13b, ...)")
        p.add_argument("--vocab", type=int, help="vocabulary of the random model")
        p.add_argument("--device", default="cuda:0", help="cuda:N (the CUDA engine) or cpu (the fp32 formulation)")
        p.add_argument("--datasets", help="comma-separated JSONL files")
        p.add_argument("--synthetic", action="store_true", help="the built-in synthetic data")
        p.add_argument("--max-examples", type=int, help="at most this many examples per file")
        p.add_argument("--max-seq-len", type=int, default=512 if sft else 256)
        p.add_argument("--template", default="chatml", choices=["chatml", "llama", "zephyr"])
        p.add_argument("--tokenizer", help="tokenizer JSON; default: UTF-8 bytes")
        p.add_argument("--epochs", type=int, default=3 if sft else 1)
        p.add_argument("--lr", type=float, default=2e-5 if sft else 5e-7)
        p.add_argument("--batch-size", type=int, default=4 if sft else 2,
                       help="sequences per micro-batch" if sft else "preference pairs per micro-batch")
        p.add_argument("--grad-accum", type=int, default=8 if sft else 16)
        if not sft:
            p.add_argument("--beta", type=float, default=0.1)
        p.add_argument("--use-lora", action="store_true", help="train low-rank adapters on the frozen model")
        p.add_argument("--lora-rank", type=int, default=64)
        p.add_argument("--lora-alpha", type=float, default=128.0)
        p.add_argument("--output", default=f"models/{name}")
        p.add_argument("--save-every", type=int, default=500 if sft else 200)
        p.add_argument("--log-every", type=int, default=10)
        p.add_argument("--seed", type=int, default=0)
        p.add_argument("--rope-theta", type=float)
        p.set_defaults(fn=fn)

    p = sp.add_parser("benchmark", help="step time / throughput of this device")
    p.add_argument("--preset", default="tiny")
    p.add_argument("--batch-size", type=int)
    p.add_argument("--seq-len", type=int)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--device")
    p.set_defaults(fn=cmd_benchmark)

    p = sp.add_parser("gpu-stress-test", help="(internal) one-step fit probe for batch calibration")
    p.add_argument("checkpoint")
    p.add_argument("--batch-size", type=int, required=True)
    p.add_argument("--seq-len", type=int, required=True)
    p.add_argument("--device")
    p.set_defaults(fn=cmd_gpu_stress_test)

    p = sp.add_parser("export-hf", help="checkpoint -> Hugging Face Qwen2ForCausalLM directory")
    p.add_argument("checkpoint", nargs="?", help="a safetensors file (or use --store)")
    p.add_argument("output_dir")
    p.add_argument("--store", help="read a stored version instead (gathers tensor-parallel shard files)")
    p.add_argument("--version", type=int, help="default: the newest stored")
    p.add_argument("--tp", type=int, default=1, help="tensor-parallel shard files per version")
    p.add_argument("--rope-theta", type=float)
    p.add_argument("--max-seq-len", type=int)
    p.set_defaults(fn=cmd_export_hf)

    p = sp.add_parser("prepare-data", help="write uint16 token shards + manifest: tokenized local text files "
                                           "(--input, --tokenizer) or uniform-random tokens (test mode)")
    p.add_argument("--output-dir", required=True)
    p.add_argument("--input", nargs="+", help=".txt (a document per line), .jsonl or .parquet files to tokenize")
    p.add_argument("--tokenizer", help="tokenizers JSON file (e.g. the Mistral v0.3 tokenizer, 32768 ids)")
    p.add_argument("--text-column", default="text", help="document field of .jsonl / .parquet inputs")
    p.add_argument("--max-samples", type=int, help="stop after this many documents")
    p.add_argument("--num-shards", type=int, default=4)
    p.add_argument("--tokens-per-shard", type=int, default=10_000_000)
    p.add_argument("--vocab", type=int, default=32768)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--upload-store")
    p.set_defaults(fn=cmd_prepare_data)

    p = sp.add_parser("micro-cluster", help="coordinator + CPU nodes on the micro-test workload")
    p.add_argument("--nodes", type=int, default=2)
    p.add_argument("--steps", type=int, default=60)
    p.add_argument("--port", type=int, default=18731)
    p.add_argument("--store")
    p.set_defaults(fn=cmd_micro_cluster)

    p = sp.add_parser("train-box", help="in-box training: every GPU of this box is one node (torch.distributed.run)")
    p.add_argument("--preset", default="tiny", help="micro-test | tiny | small | medium | large")
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--log-every", type=int, default=50)
    p.add_argument("--data-dir", help="directory of shard_XXXX.bin token shards (default: synthetic tokens)")
    p.add_argument("--shards-fraction", type=float, default=0.2, help="share of the shards each node reads")
    p.add_argument("--batch-size", type=int)
    p.add_argument("--grad-accum", type=int, help="micro-batches per optimizer step (gradient accumulation)")
    p.add_argument("--merge-sms", type=int,
                   help="SMs reserved for the merge kernels on each GPU (green-context partition; 0 = priority stream)")
    p.add_argument("--seq-len", type=int)
    p.add_argument("--push-every", type=int)
    p.add_argument("--top-k", type=float)
    p.add_argument("--no-int8", action="store_true")
    p.add_argument("--bandwidth-adaptive", action="store_true")
    p.add_argument("--lr", type=float)
    p.add_argument("--tp", type=int)
    p.add_argument("--tp-mode", default="fused", choices=["fused", "nccl"])
    p.add_argument("--activation-checkpointing", action="store_true")
    p.add_argument("--payload-slots", type=int)
    p.add_argument("--sync", default="inbox", choices=["inbox", "nccl"])
    p.add_argument("--no-push", action="store_true", help="train only (no protocol)")
    p.add_argument("--checkpoint-store", help="persist merged versions here (directory or S3 endpoint)")
    p.add_argument("--checkpoint-every", type=int)
    p.add_argument("--keep-versions", type=int)
    p.add_argument("--resume", action="store_true")
    p.add_argument("--metrics-port", type=int)
    p.add_argument("--loss-based-lr", action="store_true")
    p.add_argument("--watchdog-secs", type=float)
    p.add_argument("--swap-mode", choices=["rebase", "push_partial"])
    p.add_argument("--ef-on-swap", choices=["fold", "keep", "reset"])
    p.add_argument("--reset-optimizer", action="store_true")
    p.add_argument("--seed", type=int)
    p.add_argument("--output", help="JSONL log (rank 0)")
    p.add_argument("--pg-timeout", type=float, default=300.0)
    p.set_defaults(fn=cmd_train_box)
    return ap


def main(argv=None):
    args = build_parser().parse_args(argv)
    from .utils.tracing import setup_logging
    setup_logging(os.environ.get("DT_LOG", "info"))
    args.fn(args)


if __name__ == "__main__":
    main()
