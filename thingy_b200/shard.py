"""Row sharding of the path across GPUs (one process per GPU).

Rows are independent, so a [M, H] batch splits into contiguous row blocks,
one per rank; each rank reads its block, writes its own q / scale /
residual_out slabs, and nothing crosses NVLink. Column-major scales follow
their rows: rank r owns the [G, M_r] slab of its rows. There is no data-path
collective; torch.distributed is used only for a barrier and for the
max-over-ranks timing reduction in the benchmark.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    start: int  # first row (inclusive)
    stop: int   # last row (exclusive)

    @property
    def rows(self) -> int:
        return self.stop - self.start


def shard_rows(M: int, world: int, rank: int) -> Shard:
    """Contiguous, near-even split of M rows; the first M % world ranks get one more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    if M < 0:
        raise ValueError("M must be >= 0")
    base, extra = divmod(M, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return Shard(rank, world, start, stop)


def all_shards(M: int, world: int) -> list[Shard]:
    return [shard_rows(M, world, r) for r in range(world)]


def init_from_env(backend: str, timeout_s: float = 120.0):
    """Join the process group described by RANK / WORLD_SIZE / MASTER_* (torchrun).

    Returns (rank, world, local_rank). A short timeout makes ranks that wait
    on a rank which died end with an error instead of hanging.
    """
    import datetime
    import os

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world > 1 and not dist.is_initialized():
        kwargs = {}
        if backend == "nccl":
            import torch

            kwargs["device_id"] = torch.device("cuda", local_rank)
        dist.init_process_group(
            backend, rank=rank, world_size=world,
            timeout=datetime.timedelta(seconds=timeout_s), **kwargs,
        )
    return rank, world, local_rank


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of a per-rank scalar (e.g. a device time) over all ranks."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
