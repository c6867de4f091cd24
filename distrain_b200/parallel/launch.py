"""Process wiring of an in-box job: one process per GPU (``torch.distributed.run``), grouped into nodes.

With tensor parallelism of size T, node k is ranks [k*T, (k+1)*T): the ranks of a node share a model
replica through a ``TensorParallel`` group, and the ranks that hold the same parameter shard on every
node form the data-parallel group over which that shard's protocol (pushes, merges, swaps) runs. Without
it every rank is one node, the shape of the reference's one-node-per-GPU deployment
(node/cli/src/continuous.rs:734-961)."""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from ..config import RunConfig


@dataclass
class BoxRank:
    rank: int
    world: int
    local: int
    device: torch.device


def init_box(timeout_secs: float = 300.0) -> BoxRank:
    """Rank, world and device from the launcher's environment; the NCCL process group when world > 1."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=timeout_secs))
    return BoxRank(rank, world, local, dev)


def node_layout(world: int, tp: int):
    """(tensor-parallel size actually used, number of nodes): TP applies when it divides the world."""
    t = tp if (tp > 1 and world % tp == 0) else 1
    return t, world // t


def box_node(run: RunConfig, br: BoxRank, enable_push: bool = True, tp_mode: str = "fused",
             sync: str = "inbox"):
    """This process's ``InBoxNode``: returns (node, node_rank, n_nodes). ``sync="nccl"`` replaces the
    compressed protocol by dense NCCL averaging of the round deltas (the comparison arm)."""
    from .node import InBoxNode
    tp_size, n_nodes = node_layout(br.world, run.tp)
    tp, dp_group = None, None
    if tp_size > 1:
        from .tensor_parallel import TensorParallel
        tp_groups = [dist.new_group([k * tp_size + i for i in range(tp_size)]) for k in range(n_nodes)]
        dp_groups = [dist.new_group([k * tp_size + i for k in range(n_nodes)]) for i in range(tp_size)]
        tp = TensorParallel(tp_groups[br.rank // tp_size], br.rank % tp_size, tp_size, mode=tp_mode,
                            rows=run.micro_batch * (run.seq_len - 1), hidden=run.model.hidden_dim, device=br.device)
        dp_group = dp_groups[br.rank % tp_size]
    node_rank = br.rank // tp_size
    nccl_arm = sync == "nccl" and enable_push
    node = InBoxNode(run, rank=node_rank, world=n_nodes, device=br.device, enable_push=enable_push and not nccl_arm,
                     tp=tp, shard=br.rank % tp_size, n_shards=tp_size, dp_group=dp_group)
    if nccl_arm:
        from .nccl_baseline import NcclDenseSync
        node.sync = NcclDenseSync(node, run, node_rank, n_nodes, br.device, group=dp_group)
    return node, node_rank, n_nodes


def node_batches(run: RunConfig, node_rank: int, n_nodes: int, data_dir: Optional[str] = None,
                 shards_fraction: float = 0.2, seed: int = 0, max_resident: int = 4):
    """The batch source of one node: its deterministic share of the token shards in ``data_dir``
    (``shard_XXXX.bin``; the reference's per-node shard assignment, core/model/src/training.rs:229-270,
    with node id ``box-node-{node_rank}``), or seeded uniform-random tokens when no directory is given.
    The ranks of one tensor-parallel node get the same source. Returns (callable, description)."""
    from ..utils.data import ShardLoader, SyntheticTokens
    B, S = run.micro_batch, run.seq_len
    if not data_dir:
        return SyntheticTokens(run.model.vocab_size, B, S, seed * 1000 + 1000 + node_rank).next_batch, \
            f"synthetic uniform tokens (seed {seed * 1000 + 1000 + node_rank})"
    from ..utils.native import shard_assignment
    files = sorted(f for f in os.listdir(data_dir) if f.startswith("shard_") and f.endswith(".bin"))
    if not files:
        raise FileNotFoundError(f"no shard_XXXX.bin files in {data_dir}")
    per_node = max(1, int(round(len(files) * shards_fraction))) if n_nodes > 1 else len(files)
    idx = shard_assignment(f"box-node-{node_rank}", 0, len(files), per_node) if n_nodes > 1 else \
        list(range(len(files)))
    loader = ShardLoader([os.path.join(data_dir, files[i]) for i in idx], S, B, max_resident=max_resident)
    return loader.next_batch, f"{len(idx)} of {len(files)} shards ({[files[i] for i in idx][:4]}...)"


def data_state_key(node_rank: int) -> str:
    return f"state/box-data/node-{node_rank}.pt"


def save_data_state(store, node_rank: int, source) -> bool:
    """Store the read position of a node's batch source (``ShardLoader`` / ``SyntheticTokens`` bound
    ``next_batch``) so that a resumed job continues the node's data instead of re-reading it."""
    import io
    src = getattr(source, "__self__", None)
    st = src.state() if src is not None and hasattr(src, "state") else None
    if st is None:
        return False
    buf = io.BytesIO()
    torch.save(st, buf)
    store.put(data_state_key(node_rank), buf.getvalue())
    return True


def restore_data_state(store, node_rank: int, source) -> bool:
    import io
    src = getattr(source, "__self__", None)
    if src is None or not hasattr(src, "restore") or not store.exists(data_state_key(node_rank)):
        return False
    src.restore(torch.load(io.BytesIO(store.get(data_state_key(node_rank))), weights_only=False))
    return True
