"""Replica plumbing of the multi-GPU runs: one process per GPU (launched by torchrun, which sets
RANK, WORLD_SIZE, LOCAL_RANK and MASTER_*), each a whole model on its own slice of the images.
The forward has no collective: torch.distributed only lines the ranks up before and after a
timed region (barrier) and takes the slowest rank's time (max), so whole-job throughput is
world x per-rank images / the slowest rank's seconds ("scaling": "weak").

`backend` is "nccl" on GPUs (the benchmark) or "gloo" (host-only tests of this logic). The
process group gets a short timeout, so ranks waiting for a rank that died end with an error
instead of hanging.
"""
from __future__ import annotations

import datetime
import os


def env() -> tuple[int, int, int]:
    """(rank, world size, local rank) from the torchrun environment; (0, 1, 0) without it."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


class Replicas:
    def __init__(self, backend: str = "nccl", timeout_s: float = 120.0):
        self.rank, self.world, self.local = env()
        self.backend = backend
        self.dist = None
        if self.world > 1:
            import torch
            import torch.distributed as dist

            kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
            if backend == "nccl":
                kwargs["device_id"] = torch.device("cuda", self.local)
            dist.init_process_group(backend, **kwargs)
            self.dist = dist

    def _tensor(self, values, dtype):
        import torch

        device = "cuda" if self.backend == "nccl" else "cpu"
        return torch.tensor(values, dtype=dtype, device=device)

    def _sync_device(self):
        if self.backend == "nccl":
            import torch

            torch.cuda.synchronize()

    def barrier(self) -> None:
        """Every rank reaches this point (and its device is idle) before any leaves it."""
        if self.dist is not None:
            import torch

            self.dist.all_reduce(self._tensor([0.0], torch.float32))
        self._sync_device()

    def max(self, value: float) -> float:
        """The largest `value` over the ranks (the slowest rank's time)."""
        if self.dist is None:
            return float(value)
        import torch

        t = self._tensor([float(value)], torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def first_image(self, per_rank: int) -> int:
        """Index of this rank's first image in the job's image sequence (rank r takes images
        r*per_rank .. r*per_rank + per_rank - 1)."""
        return self.rank * per_rank

    def share(self, total: int) -> int:
        """This rank's part of `total` items: total // world, the remainder going one each to the
        first ranks, so the parts add up to `total`."""
        return total // self.world + (1 if self.rank < total % self.world else 0)

    def throughput(self, per_rank_items: float, slowest_seconds: float) -> float:
        """Whole-job items per second: every rank's items over the slowest rank's time."""
        return self.world * per_rank_items / slowest_seconds

    def close(self) -> None:
        if self.dist is not None:
            self.barrier()
            self.dist.destroy_process_group()
            self.dist = None
