"""Replica (data-parallel) plumbing for one process per GPU.

Images are independent, so a multi-GPU run is N replicas of the engine, one
per GPU, each processing its own images; there is no collective on the data
path.  `torch.distributed` is used only for the control plane: a barrier
around timed regions, the max over ranks of a device time, and ordering the
one-time creation of a shared model file.  These helpers hold that logic so
the benchmark and the tests (gloo ranks on CPU) run the same code.

    info = RankInfo.from_env()
    with ProcessGroup(info, backend="nccl") as pg:
        lo, hi = shard(global_batch, info.rank, info.world)
        ...
        t = pg.max_over_ranks(local_ms)
"""
from __future__ import annotations

import dataclasses
import datetime
import os
from typing import Callable, Optional


@dataclasses.dataclass(frozen=True)
class RankInfo:
    rank: int = 0
    world: int = 1
    local_rank: int = 0

    @staticmethod
    def from_env(env=None) -> "RankInfo":
        env = os.environ if env is None else env
        world = int(env.get("WORLD_SIZE", "1"))
        rank = int(env.get("RANK", "0"))
        local = int(env.get("LOCAL_RANK", str(rank)))
        if world < 1 or not 0 <= rank < world or local < 0:
            raise ValueError(f"bad rank environment: RANK={rank} WORLD_SIZE={world} LOCAL_RANK={local}")
        return RankInfo(rank, world, local)


def shard(n_items: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous split of n_items over `world` ranks: [lo, hi) of `rank`.

    The first n_items % world ranks get one extra item, so every item is
    owned by exactly one rank and sizes differ by at most one.
    """
    if world < 1 or not 0 <= rank < world or n_items < 0:
        raise ValueError("bad shard arguments")
    base, extra = divmod(n_items, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


class ProcessGroup:
    """The default process group for `info` (no-op when world == 1).

    `backend` is "nccl" on GPUs ("gloo" in CPU tests).  The timeout is short
    so that ranks waiting on a rank that died end with an error instead of
    hanging.
    """

    def __init__(self, info: RankInfo, backend: str = "nccl", timeout_s: float = 300.0,
                 device: Optional[object] = None):
        self.info = info
        self.backend = backend
        self.device = device
        self._dist = None
        if info.world > 1:
            import torch.distributed as dist
            kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
            if backend == "nccl" and device is not None:
                kw["device_id"] = device
            dist.init_process_group(backend, rank=info.rank, world_size=info.world, **kw)
            self._dist = dist

    def __enter__(self) -> "ProcessGroup":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def close(self) -> None:
        if self._dist is not None:
            self._dist.destroy_process_group()
            self._dist = None

    def barrier(self) -> None:
        if self._dist is not None:
            self._dist.barrier()

    def max_over_ranks(self, value: float) -> float:
        """Max of a per-rank scalar (a device time) over all ranks."""
        if self._dist is None:
            return float(value)
        import torch
        dev = self.device if self.backend == "nccl" else "cpu"
        t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
        self._dist.all_reduce(t, op=self._dist.ReduceOp.MAX)
        return float(t.item())

    def gather_to_rank0(self, value: float) -> Optional[list]:
        """Every rank's scalar, on rank 0 (None elsewhere)."""
        if self._dist is None:
            return [float(value)]
        import torch
        dev = self.device if self.backend == "nccl" else "cpu"
        t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
        out = [torch.zeros_like(t) for _ in range(self.info.world)]
        self._dist.all_gather(out, t)
        return [float(x.item()) for x in out] if self.info.rank == 0 else None


def create_once(path: str, make: Callable[[str], None], pg: ProcessGroup) -> str:
    """Rank 0 creates `path` (atomically, via a temporary name) if it is
    missing; the other ranks wait at a barrier and then see the finished file."""
    if pg.info.rank == 0 and not os.path.exists(path):
        tmp = f"{path}.tmp{os.getpid()}"
        make(tmp)
        os.replace(tmp, path)
    pg.barrier()
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    return path
