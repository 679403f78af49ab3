"""Batch sharding across GPUs (one process per GPU) for the sparse-attention path.

The reference runs on one device (``world_size = 1`` and ``rank = 0`` are
hard-coded, reference/task2_v0_ref.py:16-17). Every operator of the path is
independent across the batch dimension -- kv[b] / kv_cache[b] belong to batch
b only -- so N GPUs each run their own slice of the batch with no collective on
the data path. torch.distributed (NCCL over NVLink on GPUs, gloo on CPU) is used
only to assemble outputs and to take the max of per-rank timings.
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def env_world() -> tuple[int, int, int]:
    """(world_size, rank, local_rank) from the torchrun environment."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str | None = None, timeout_s: float = 120.0) -> tuple[int, int, int]:
    """Initialises the default process group when WORLD_SIZE > 1.

    backend defaults to "nccl" when CUDA is available, else "gloo". A short
    timeout makes ranks that wait for a failed peer end with an error.
    """
    world, rank, local = env_world()
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kwargs = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s), **kwargs)
    return world, rank, local


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the contiguous slice of n items owned by `rank`.

    The first n % world ranks get one extra item, so every item is owned by
    exactly one rank and slices differ by at most one.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_batch(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's slice of `t` along dim 0 (a view, no copy)."""
    a, b = shard_range(t.shape[0], rank, world)
    return t[a:b]


def gather_batch(shard: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """Concatenates every rank's batch slice (as produced by shard_range) on
    every rank. Equal slices use one all_gather_into_tensor; unequal ones pad
    to the largest slice and trim."""
    world = dist.get_world_size(group)
    if (dist.get_backend(group) == "gloo" and shard.element_size() == 2 and shard.dim() > 1
            and shard.shape[-1] % 2 == 0):
        # gloo has no 16-bit collectives: move bf16/int16 payloads as int32 pairs
        out = gather_batch(shard.contiguous().view(torch.int32), n_total, group)
        return out.view(shard.dtype)
    sizes = [shard_range(n_total, r, world) for r in range(world)]
    width = max(b - a for a, b in sizes)
    if shard.shape[0] != width:
        pad = torch.zeros((width - shard.shape[0],) + tuple(shard.shape[1:]), dtype=shard.dtype,
                          device=shard.device)
        shard = torch.cat([shard, pad])
    full = torch.empty((world * width,) + tuple(shard.shape[1:]), dtype=shard.dtype,
                       device=shard.device)
    dist.all_gather_into_tensor(full, shard.contiguous(), group=group)
    if all(b - a == width for a, b in sizes):
        return full
    return torch.cat([full[r * width:r * width + (b - a)] for r, (a, b) in enumerate(sizes)])


def max_over_ranks(x: float, group=None) -> float:
    """Max of a per-rank scalar (timings are reported as the slowest rank)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return x
    dev = torch.device("cuda", torch.cuda.current_device()) if (
        dist.get_backend(group) == "nccl") else torch.device("cpu")
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def barrier(group=None) -> None:
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.barrier(group=group)
