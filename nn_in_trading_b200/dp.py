"""Data-parallel plumbing: one process per GPU, launched by torchrun.

Host-side coordination (rendezvous, the NCCL unique id, barriers and the max
of per-rank timings) goes through torch.distributed; the gradient exchange
itself is the library's own NCCL allreduce inside nn_dp_update_begin/end
(one allreduce of the flat weight-gradient arena per step, averaged over the
ranks, then the reference update arithmetic on every rank).

Partitioning is the batch: every rank trains its own shard of independent
samples (sequences, series, transitions), so the mean of the ranks'
batch-mean gradients equals the batch-mean gradient of the whole global
batch when the shards are equal.
"""
from __future__ import annotations

import datetime
import os


def env_rank() -> tuple[int, int, int]:
    """(rank, world, local_rank) from the torchrun environment (defaults: single process)."""
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", rank))
    return rank, world, local


def init_host_group(backend: str = "gloo", timeout_s: int = 300):
    """Process group for host-side coordination (MASTER_ADDR/PORT from the environment)."""
    import torch.distributed as dist
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def share_unique_id(uid: bytes | None, rank: int) -> bytes:
    """Broadcast rank 0's 128-byte NCCL unique id to every rank."""
    import torch.distributed as dist
    box = [uid if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    if not isinstance(box[0], (bytes, bytearray)) or len(box[0]) != 128:
        raise RuntimeError("bad NCCL unique id received")
    return bytes(box[0])


def max_over_ranks(value: float) -> float:
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([float(value)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shard(total: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of rank's equal shard of `total` samples (total must divide evenly)."""
    if total % world:
        raise ValueError(f"batch {total} does not split evenly over {world} ranks")
    n = total // world
    return rank * n, (rank + 1) * n


def join_dp(ctx, rank: int, world: int) -> None:
    """Create the library's NCCL communicator on every rank (collective)."""
    uid = share_unique_id(ctx.dp_unique_id() if rank == 0 else None, rank)
    ctx.dp_init(rank, world, uid)
