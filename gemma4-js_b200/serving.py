"""Batched decode serving over independent replicas, one process per GPU.

Decode sequences are independent, so the batch is split across the GPUs of a box with
no collective on the data path: each rank owns a contiguous block of sequences, a full
copy of the weights and the KV caches of its sequences, and runs its decode step as one
CUDA graph.  The only exchange is the gather of the step's token ids to every rank
(NCCL over NVLink on GPUs; gloo in CPU tests), so rank 0 can stream or stop.

The reference has no multi-GPU code; this is the partitioning of the serving config.
A rank that dies or never joins surfaces as an error on the others when the process
group's timeout ends their next collective, never as a hang; with a `StepHeartbeat`
the others learn of it on the host, between steps, before they launch anything more.
"""
from __future__ import annotations

import datetime
import time

import torch


def partition(total: int, world: int, rank: int) -> tuple[int, int]:
    """Sequences [start, start + count) of `rank`: a contiguous, balanced split of
    `total` over `world` ranks (the first total % world ranks get one more)."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"partition({total}, {world}, {rank})")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def init_process_group(backend: str, timeout_s: float = 120.0, device: torch.device | None = None):
    """torch.distributed init from the torchrun environment with a short timeout."""
    import torch.distributed as dist
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
    return dist


class TokenGather:
    """Gathers each rank's step token ids into one [total] tensor, in sequence order."""

    def __init__(self, dist, total: int, device):
        self.dist = dist
        self.world = dist.get_world_size() if dist is not None else 1
        self.total = total
        self.counts = [partition(total, self.world, r)[1] for r in range(self.world)]
        self.pad = max(self.counts)
        self.bufs = [torch.empty(self.pad, dtype=torch.int32, device=device) for _ in range(self.world)]
        self.local = torch.empty(self.pad, dtype=torch.int32, device=device)
        self.out = torch.empty(total, dtype=torch.int32, device=device)

    def gather(self, local_ids: torch.Tensor) -> torch.Tensor:
        n = local_ids.numel()
        if self.world == 1:
            self.out[:n].copy_(local_ids)
            return self.out
        self.local[:n].copy_(local_ids)
        self.dist.all_gather(self.bufs, self.local)
        off = 0
        for r, c in enumerate(self.counts):
            self.out[off:off + c].copy_(self.bufs[r][:c])
            off += c
        return self.out


class RankFailure(RuntimeError):
    """A peer rank stopped stepping (it died, hung or left the job)."""


class StepHeartbeat:
    """Host-side liveness between decode steps over a c10d key-value store (the process
    group's TCPStore, or any `torch.distributed.Store`).  Each rank calls `enter(step)`
    before launching a step: it announces the step and returns once every peer has
    announced it too, or raises RankFailure naming the ranks that did not within
    `timeout_s` -- so a rank that left between steps is reported before the others
    enqueue a kernel or a collective that would wait for it."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 2.0, prefix: str = "g4hb"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _announced(self, r: int) -> int:
        if not self.store.check([self._key(r)]):
            return -1
        return int(self.store.get(self._key(r)).decode())

    def enter(self, step: int) -> None:
        self.store.set(self._key(self.rank), str(step))
        deadline = time.monotonic() + self.timeout_s
        behind = [r for r in range(self.world) if r != self.rank]
        while True:
            behind = [r for r in behind if self._announced(r) < step]
            if not behind:
                return
            if time.monotonic() > deadline:
                raise RankFailure(f"rank {self.rank}: rank(s) {behind} did not reach step {step} "
                                  f"within {self.timeout_s:.1f} s")
            time.sleep(0.002)
