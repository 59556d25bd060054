"""Per-GPU shard split and host-side coordination of a multi-GPU job.

One process per GPU (launched by torchrun or any launcher that sets RANK,
WORLD_SIZE, MASTER_ADDR and MASTER_PORT).  The FHE NTT path shards with no
data exchange: each rank owns a contiguous range of ciphertexts (or of RNS
limbs), generates its inputs from global indices (bc_fill_uniform with
first_poly / total_polys), transforms them on its own GPU and exchanges only
64-bit digests for verification.  The reference has no collective on this
path either; its nearest analog is GpuPool::parallel_map, which
round-robins whole ops over devices
(crates/barracuda/src/multi_gpu/gpu_pool.rs:194-231).

Failure detection happens on the host.  Every rank posts a status for each
step under a key of the process group's store (ok, or the error it hit),
and before the next collective every rank waits for its peers' keys with a
deadline.  A rank that raised, exited or never joined therefore surfaces as
ShardFailure on the others instead of a hang inside a collective; the
process group's own timeout is the last bound.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta
from typing import List, Optional, Sequence

from .plan import partition

MASK64 = (1 << 64) - 1


class ShardFailure(RuntimeError):
    """A peer rank failed a step or stopped answering."""

    def __init__(self, rank: int, message: str):
        super().__init__(f"rank {rank}: {message}")
        self.rank = rank
        self.message = message


@dataclass(frozen=True)
class Shard:
    """The units (ciphertexts or limbs) rank `rank` of `world` owns."""
    rank: int
    world: int
    total: int
    begin: int
    count: int

    @classmethod
    def of(cls, total: int, world: int, rank: int) -> "Shard":
        begin, count = partition(total, world, rank)
        return cls(rank, world, total, begin, count)


def job_digest(shard_digests: Sequence[int]) -> int:
    """Digest of the whole job from per-shard digests taken with global
    first indices (bc_digest): their sum mod 2^64."""
    return sum(int(d) for d in shard_digests) & MASK64


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


class ShardGroup:
    """Process group of a sharded job plus the status exchange above.

    backend: "nccl" (GPUs) or "gloo" (CPU tests); world_size 1 needs no
    process group at all.  `timeout` bounds the rendezvous, every status
    wait and the process group's collectives.
    """

    def __init__(self, backend: str = "nccl", timeout: float = 60.0, device=None):
        import torch.distributed as dist

        self.dist = dist
        self.rank = _env_int("RANK", 0)
        self.world = _env_int("WORLD_SIZE", 1)
        self.timeout = timeout
        self.backend = backend
        self.device = device
        self.store = None
        self._own_pg = False
        if self.world == 1:
            return
        if not dist.is_initialized():
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            kw = {"device_id": device} if (backend == "nccl" and device is not None) else {}
            try:
                dist.init_process_group(backend, init_method="env://", rank=self.rank,
                                        world_size=self.world, timeout=timedelta(seconds=timeout), **kw)
            except Exception as e:  # a peer never joined, or the master is gone
                raise ShardFailure(-1, f"rendezvous of {self.world} ranks failed: {e}") from e
            self._own_pg = True
        # The statuses live in the default group's store (the one torchrun or
        # env:// rendezvous created), under their own prefix.
        self.store = dist.PrefixStore("barracuda_shard", dist.distributed_c10d._get_default_store())

    # ---------------------------------------------------------- statuses
    def post(self, step: str, error: Optional[str] = None) -> None:
        """Publishes this rank's outcome of `step` (None: success)."""
        if self.store is not None:
            self.store.set(f"{step}/{self.rank}", "ok" if error is None else "err:" + error)

    def check(self, step: str, timeout: Optional[float] = None) -> None:
        """Waits until every peer posted `step`; raises ShardFailure for the
        first peer that reported an error or posted nothing in time."""
        if self.store is None:
            return
        t = timedelta(seconds=self.timeout if timeout is None else timeout)
        for r in range(self.world):
            if r == self.rank:
                continue
            key = f"{step}/{r}"
            try:
                self.store.wait([key], t)
            except Exception as e:
                raise ShardFailure(r, f"no status for step '{step}' within {t.total_seconds():g} s") from e
            v = self.store.get(key).decode()
            if v != "ok":
                raise ShardFailure(r, v[4:] if v.startswith("err:") else v)

    def step(self, name: str, fn, *args, **kwargs):
        """Runs fn on this rank, posts its outcome, then checks the peers:
        every rank learns of a failure anywhere before the next collective."""
        try:
            out = fn(*args, **kwargs)
        except Exception as e:
            self.post(name, f"{type(e).__name__}: {e}")
            raise
        self.post(name)
        self.check(name)
        return out

    # ------------------------------------------------------- collectives
    def _tensor(self, values: Sequence[int]):
        import torch
        signed = [v - (1 << 64) if v >= (1 << 63) else v for v in (int(x) & MASK64 for x in values)]
        dev = self.device if (self.backend == "nccl" and self.device is not None) else "cpu"
        return torch.tensor(signed, dtype=torch.int64, device=dev)

    def gather_u64(self, values: Sequence[int]) -> List[List[int]]:
        """All ranks' `values` (same length everywhere), as unsigned ints."""
        if self.world == 1:
            return [[int(v) & MASK64 for v in values]]
        t = self._tensor(values)
        parts = [t.clone() for _ in range(self.world)]
        self.dist.all_gather(parts, t)
        return [[int(v) & MASK64 for v in p.cpu().tolist()] for p in parts]

    def max_f64(self, value: float) -> float:
        """Maximum of a float over the ranks (device times: max over ranks)."""
        if self.world == 1:
            return float(value)
        import torch
        dev = self.device if (self.backend == "nccl" and self.device is not None) else "cpu"
        t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def barrier(self) -> None:
        if self.world > 1:
            self.dist.barrier()

    def close(self) -> None:
        if self._own_pg and self.dist.is_initialized():
            self.dist.destroy_process_group()
        self._own_pg = False
