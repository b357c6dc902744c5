"""Independent decode streams spread over the GPUs of one node, one process per GPU.

Streams never interact (each has its own cache rows; attention and eviction are per
(batch, head)), so the work partitions with no exchange on the hot path: rank r takes a
contiguous block of the streams.  torch.distributed (NCCL on GPUs, gloo on CPU) is used
only around the measured region -- a barrier, the max of the per-rank times, and the
sums of per-rank results (NLL sums, token counts).
"""

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def shard(n_streams: int, rank: int, world: int) -> range:
    """Streams [start, stop) of `rank`: contiguous blocks, the first n % world ranks one
    stream larger.  Every stream keeps its global index (and so its seed) at any world size."""
    if world < 1 or not 0 <= rank < world or n_streams < 0:
        raise ValueError(f"bad partition: {n_streams} streams, rank {rank} of {world}")
    base, extra = divmod(n_streams, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def init_from_env(backend: str, timeout_s: float = 120.0) -> tuple[int, int, int]:
    """(rank, world, local_rank) from torchrun's environment; initialises the process group
    when world > 1 with a short timeout so a lost rank ends the others with an error."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world > 1 and not dist.is_initialized():
        kwargs = {}
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s),
                                **kwargs)
    return rank, world, local


def _device() -> torch.device:
    if dist.is_initialized() and dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def barrier() -> None:
    if dist.is_initialized():
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def reduce_max(x: float) -> float:
    """Max over ranks (the job's time is its slowest rank's)."""
    if not dist.is_initialized():
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(values: list[float]) -> list[float]:
    """Elementwise sum over ranks."""
    if not dist.is_initialized():
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.tolist()


def shutdown() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
