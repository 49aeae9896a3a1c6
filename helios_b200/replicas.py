"""One engine replica per GPU: process-group plumbing for measurement only.

The packed tick has no cross-GPU exchange (a Qwen3-4B replica fits one B200),
so requests are sharded round-robin across ranks and nothing on the data path
talks to another GPU. The process group exists to line the ranks up (barrier)
and to take the maximum of their timings. Rendezvous uses 127.0.0.1.
"""

from __future__ import annotations

import os
from collections.abc import Sequence
from datetime import timedelta

import torch
import torch.distributed as dist


def world() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment (1 process if unset)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def init(backend: str, timeout_s: float = 120.0) -> bool:
    rank, size, _ = world()
    if size <= 1:
        return False
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if backend == "nccl":
        # NCCL's own log goes to stderr, so rank 0's stdout carries only what the caller prints.
        # At NCCL_DEBUG=VERSION (this image's default) NCCL prints its version banner to stdout
        # whatever NCCL_DEBUG_FILE says; from WARN up the banner and warnings go to that file.
        if os.environ.get("NCCL_DEBUG", "").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    dist.init_process_group(backend=backend, rank=rank, world_size=size, timeout=timedelta(seconds=timeout_s))
    return True


def shard(items: Sequence, rank: int, size: int) -> list:
    """Round-robin share of ``items`` for ``rank`` (request streams to replicas)."""
    return list(items[rank::size])


def barrier(device: torch.device | None = None) -> None:
    if dist.is_available() and dist.is_initialized():
        if device is not None and device.type == "cuda" and dist.get_backend() == "nccl":
            dist.barrier(device_ids=[device.index])
        else:
            dist.barrier()


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return value
    use = device if (device is not None and dist.get_backend() == "nccl") else torch.device("cpu")
    t = torch.tensor([value], dtype=torch.float64, device=use)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device: torch.device | None = None) -> float:
    if not (dist.is_available() and dist.is_initialized()):
        return value
    use = device if (device is not None and dist.get_backend() == "nccl") else torch.device("cpu")
    t = torch.tensor([value], dtype=torch.float64, device=use)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_objects(value, device: torch.device | None = None) -> list:
    """Every rank's ``value`` (picklable host data: per-replica results such as token counts
    and time-to-first-token samples), in rank order, on every rank. Measurement plumbing on
    the host, not a data-path exchange."""
    if not (dist.is_available() and dist.is_initialized()):
        return [value]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, value)
    return out


def shutdown() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
