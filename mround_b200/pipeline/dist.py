"""Data-parallel plumbing: one process per GPU, NCCL over NVLink.

The tuning loop shards naturally over calibration sequences (the reference's
micro-batch contract, mround/pipeline/runner.py:984-1044): rank ``r`` of ``N``
holds sequences ``j`` with ``j % N == r`` of every batch, for both activation
streams.  Per step the ranks exchange only (a) three 2048-bin histograms for
the exact global outlier threshold and (b) the float32 weight gradients:
reduce-scattered by rows, each rank applying the signed step to its own rows
and all-gathering the updated bf16 operands (or, where a weight's rows do not
divide by the rank count, all-reduced and applied on every rank).

``DistContext`` wraps ``torch.distributed`` with a bounded timeout; with one
rank every call is a no-op.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as tdist

__all__ = ["DistContext", "init_from_env"]


class DistContext:
    def __init__(self, rank: int = 0, world: int = 1, group=None) -> None:
        self.rank = rank
        self.world = world
        self.group = group

    @property
    def active(self) -> bool:
        return self.world > 1

    def shard(self, batch_size: int) -> list[int]:
        """Sequence indices of a batch this rank holds."""
        return [j for j in range(batch_size) if j % self.world == self.rank]

    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            tdist.all_reduce(t, group=self.group)
        return t

    def all_reduce_async(self, t: torch.Tensor):
        if self.world > 1:
            return tdist.all_reduce(t, group=self.group, async_op=True)
        return None

    def reduce_scatter_async(self, out: torch.Tensor, full: torch.Tensor):
        """Sum ``full`` over ranks; this rank receives its contiguous 1/N in ``out``."""
        if self.world > 1:
            return tdist.reduce_scatter_tensor(out, full, group=self.group, async_op=True)
        out.copy_(full)
        return None

    def all_gather_async(self, full: torch.Tensor, part: torch.Tensor):
        """Concatenate every rank's ``part`` (rank order) into ``full``."""
        if self.world > 1:
            return tdist.all_gather_into_tensor(full, part, group=self.group, async_op=True)
        full.copy_(part)
        return None

    def barrier(self) -> None:
        if self.world > 1:
            tdist.barrier(group=self.group)

    def max_scalar(self, value: float, device) -> float:
        if self.world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX, group=self.group)
        return float(t.item())


def init_from_env(backend: str | None = None, timeout_s: float = 300.0) -> DistContext:
    """Initialise from torchrun's RANK/WORLD_SIZE (127.0.0.1 rendezvous)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return DistContext()
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    rank = int(os.environ["RANK"])
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    if not tdist.is_initialized():
        tdist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
    return DistContext(rank, world, None)


def shutdown() -> None:
    """Destroy the process group (``init_from_env``'s), if one is open."""
    if tdist.is_available() and tdist.is_initialized():
        tdist.destroy_process_group()
