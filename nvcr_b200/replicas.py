"""Multi-GPU plumbing for the exact-convolution path: one process per GPU
(torchrun), independent replicas, no collective on the data path.

The path does not shard within a stage. Independent streams do: stream s runs
on rank s mod world (round-robin), each rank with its own executor and
weights. The only cross-rank traffic is a barrier around timed regions, one
max-reduction of the elapsed time, so the slowest rank sets the number, and a
sum of the outputs each rank found differing from the reference's digests.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass


@dataclass(frozen=True)
class RankEnvironment:
    world: int
    rank: int
    local: int


def rank_environment() -> RankEnvironment:
    """WORLD_SIZE, RANK and LOCAL_RANK as torchrun sets them (1, 0, 0 without it)."""
    return RankEnvironment(int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
                           int(os.environ.get("LOCAL_RANK", "0")))


def streams_of(rank: int, world: int, streams: int) -> list[int]:
    """The streams rank `rank` decodes: s with s mod world == rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return [s for s in range(streams) if s % world == rank]


class Group:
    """Barrier and max-over-ranks for the timed regions. A world of one needs no
    process group; otherwise `backend` is "nccl" (one GPU per rank) or "gloo"
    (CPU, for tests), with a short timeout so that ranks waiting on a dead peer
    end with an error instead of hanging."""

    def __init__(self, env: RankEnvironment, backend: str = "nccl", device=None, timeout_s: int = 120) -> None:
        self.env = env
        self.device = device
        self._dist = None
        if env.world > 1:
            import torch.distributed as dist

            kwargs = {"device_id": device} if backend == "nccl" and device is not None else {}
            dist.init_process_group(backend, rank=env.rank, world_size=env.world,
                                    timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
            self._dist = dist

    def barrier(self) -> None:
        if self._dist is not None:
            self._dist.barrier()

    def max(self, value: float) -> float:
        if self._dist is None:
            return value
        import torch

        t = torch.tensor([value], dtype=torch.float64, device=self.device if self.device is not None else "cpu")
        self._dist.all_reduce(t, op=self._dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, value: float) -> float:
        if self._dist is None:
            return value
        import torch

        t = torch.tensor([value], dtype=torch.float64, device=self.device if self.device is not None else "cpu")
        self._dist.all_reduce(t, op=self._dist.ReduceOp.SUM)
        return float(t.item())

    def close(self) -> None:
        if self._dist is not None:
            self._dist.destroy_process_group()
            self._dist = None
