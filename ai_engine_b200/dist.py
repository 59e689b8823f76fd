"""Multi-GPU plumbing for the conv path: one process per GPU.

Frames (or video streams) are independent, so each rank processes its own
contiguous slice of the batch with no collective on the hot path.  The
collectives here are off the hot path: the max-over-ranks of a timing, and
the optional gather of every rank's outputs into one buffer on the root
(NCCL over NVLink on GPUs, gloo on CPU), for callers that want a single
host buffer.
"""
from __future__ import annotations

import datetime
import os
from typing import Optional, Tuple

import torch
import torch.distributed as dist


def env_rank() -> Tuple[int, int, int]:
    """(rank, local_rank, world_size) from torchrun's environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def init(backend: str = "nccl", timeout_s: float = 120.0, device: Optional[torch.device] = None):
    """Initialise the process group (short timeout: ranks waiting on a dead
    peer fail instead of hanging)."""
    if dist.is_initialized():
        return
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if backend == "nccl" and device is not None:
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)


def gpu_local_cpus(device_index: int, nvml=None) -> Optional[list]:
    """The host CPUs NVML reports as closest to GPU `device_index` (its
    NUMA node's cores), or None when NVML cannot tell.  `nvml` is the
    pynvml module (a stand-in in tests)."""
    try:
        if nvml is None:
            import pynvml as nvml
        nvml.nvmlInit()
        h = nvml.nvmlDeviceGetHandleByIndex(device_index)
        words = (os.cpu_count() + 63) // 64
        mask = nvml.nvmlDeviceGetCpuAffinity(h, words)
        cpus = [64 * i + b for i, wd in enumerate(mask) for b in range(64) if (int(wd) >> b) & 1]
        return [c for c in cpus if c < os.cpu_count()] or None
    except Exception:
        return None


def bind_to_gpu_numa(device_index: int, nvml=None) -> Optional[list]:
    """Pin this process to the CPUs local to its GPU before it allocates
    pinned host buffers, so their pages are placed on the GPU's NUMA node
    (first touch) and each rank's host<->device copies use its own socket's
    memory.  With one process per GPU on a two-socket host, unbound ranks
    place every rank's staging buffers wherever the scheduler ran them.
    Returns the CPU list, or None (nothing changed) when it is unknown."""
    cpus = gpu_local_cpus(device_index, nvml)
    if cpus:
        try:
            os.sched_setaffinity(0, cpus)
        except OSError:
            return None
    return cpus


def shard_range(n_total: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [start, end) slice of n_total frames for `rank`; the first
    n_total % world ranks take one extra frame."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(n_total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(value: float, device=None) -> float:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_outputs(local: torch.Tensor, n_total: int, root: int = 0) -> Optional[torch.Tensor]:
    """Gather every rank's output slice [n_r, ...] into one [n_total, ...]
    tensor on `root` (rank order = batch order).  Slices are padded to the
    largest shard so one all_gather moves everything; other ranks get None."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return local
    world, rank = dist.get_world_size(), dist.get_rank()
    counts = [shard_range(n_total, r, world) for r in range(world)]
    cap = max(e - s for s, e in counts)
    padded = local.new_zeros((cap,) + tuple(local.shape[1:]))
    padded[: local.shape[0]].copy_(local)
    full = local.new_empty((world * cap,) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(full, padded)
    if rank != root:
        return None
    parts = [full[r * cap: r * cap + (e - s)] for r, (s, e) in enumerate(counts)]
    return torch.cat(parts, 0)
