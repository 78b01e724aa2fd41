"""Peer slot buffers of the fused GEMM -> reduce-scatter (one process per GPU).

Every rank allocates one device pool holding, for each fused weight, ``world``
source slots of its own rows (``rows / world`` x ``cols`` float32 each) and,
at the end, one int64 flag per (weight, source).  The pools are exported as
CUDA IPC handles (``mr_ipc_export``), exchanged once over the process group
(``all_gather_object``) and mapped on every other rank (``mr_ipc_import``), so
that a rank's weight-gradient GEMM (``mr_gemm_rs``) stores each row directly
into its owner's slot for this source and releases the step's epoch into the
owner's flag, and the owner sums its slots in rank order (``mr_reduce_slots``).

With ``copy_engine``, the GEMM instead writes the whole gradient locally and
the copy engines move each owner's rows (``mr_peer_send``: one
cudaMemcpyAsync per owner on that owner's stream, then a one-thread kernel
releasing the epoch), so no SM stores to peer memory and the transfer overlaps
the rest of the backward.  The owner's sum is the same ``mr_reduce_slots``.

One allocation per rank means one handle per peer mapping.  Mappings are
closed by :meth:`PeerExchange.close`.  No multicast object is involved.
"""

from __future__ import annotations

import ctypes
import dataclasses

import torch
import torch.distributed as tdist

from mround_b200 import kernels
from mround_b200._native import check, lib
from mround_b200.pipeline.dist import DistContext

__all__ = ["LayerExchange", "PeerExchange"]


@dataclasses.dataclass
class LayerExchange:
    """What one fused weight's GEMM and its owner-side sum need."""

    rows_per_rank: int
    cols: int
    dst_ptrs: list[int]    # rank o's slot for this source, for every o
    flag_ptrs: list[int]   # rank o's flag for this source, for every o
    slots: torch.Tensor    # this rank's (world, rows_per_rank, cols) source slots
    flags: torch.Tensor    # this rank's (world,) flags, one per source
    done: torch.Tensor     # this rank's CTA counter (int32, zero between launches)
    epoch: int = 0
    active: bool = False
    streams: list | None = None  # copy-engine mode: one stream per owner rank
    copy_events: list = dataclasses.field(default_factory=list)

    @property
    def copy_engine(self) -> bool:
        return self.streams is not None

    def send(self, grad: torch.Tensor) -> None:
        """Copy-engine mode: after the current stream's work so far (the GEMM
        that wrote ``grad``, the full float32 gradient), move each owner's rows
        into its slot for this rank and release the epoch into its flag."""
        ready = torch.cuda.Event()
        ready.record()
        self.copy_events = []
        per = self.rows_per_rank
        for owner, stream in enumerate(self.streams):
            stream.wait_event(ready)
            with torch.cuda.stream(stream):
                kernels.peer_send(self.dst_ptrs[owner], grad[owner * per:(owner + 1) * per],
                                  self.flag_ptrs[owner], self.epoch)
                done = torch.cuda.Event()
                done.record(stream)
            self.copy_events.append(done)

    def wait_copies(self) -> None:
        """Order the current stream after this rank's copies (its own flag is
        then set, and the gradient buffer may be written again)."""
        stream = torch.cuda.current_stream()
        for event in self.copy_events:
            stream.wait_event(event)
        self.copy_events = []


class PeerExchange:
    def __init__(self, dist: DistContext, shapes: list[tuple[int, int]],
                 device: torch.device, *, copy_engine: bool = False) -> None:
        """``shapes``: (rows, cols) of each fused weight, rows divisible by the
        rank count, cols by 4.  Collective: every rank calls it in the same order."""
        world, rank = dist.world, dist.rank
        self.streams = ([torch.cuda.Stream(device) for _ in range(world)] if copy_engine
                        else None)
        self.world, self.rank = world, rank
        offsets, total = [], 0
        for rows, cols in shapes:
            offsets.append(total)
            total += rows * cols  # world slots of rows/world rows each
        flag_off = (total + 3) // 4 * 4
        total = flag_off + 2 * world * len(shapes)  # int64 flags as pairs of floats
        self.pool = torch.zeros(total, dtype=torch.float32, device=device)
        self.done = torch.zeros(len(shapes), dtype=torch.int32, device=device)
        flags_all = self.pool[flag_off:].view(torch.int64).view(len(shapes), world)

        handle = (ctypes.c_uint8 * int(lib().mr_ipc_handle_bytes()))()
        off = ctypes.c_int64(0)
        check(lib().mr_ipc_export(self.pool.data_ptr(), ctypes.cast(handle, ctypes.c_void_p),
                                  ctypes.byref(off)), "mr_ipc_export")
        mine = (bytes(handle), int(off.value))
        gathered: list = [None] * world
        tdist.all_gather_object(gathered, mine, group=dist.group)
        self._bases: list[int] = []
        pool_ptrs = []
        for r, (h, o) in enumerate(gathered):
            if r == rank:
                pool_ptrs.append(self.pool.data_ptr())
                continue
            hb = (ctypes.c_uint8 * len(h)).from_buffer_copy(h)
            base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
            check(lib().mr_ipc_import(ctypes.cast(hb, ctypes.c_void_p), o, ctypes.byref(base),
                                      ctypes.byref(ptr)), "mr_ipc_import")
            self._bases.append(base.value)
            pool_ptrs.append(ptr.value)
        self.layers: list[LayerExchange] = []
        for i, ((rows, cols), start) in enumerate(zip(shapes, offsets)):
            per = rows // world
            slot_bytes = per * cols * 4
            slots = self.pool[start:start + rows * cols].view(world, per, cols)
            dst = [pool_ptrs[o] + start * 4 + rank * slot_bytes for o in range(world)]
            flag = [pool_ptrs[o] + flag_off * 4 + (i * world + rank) * 8 for o in range(world)]
            self.layers.append(LayerExchange(per, cols, dst, flag, slots, flags_all[i],
                                             self.done[i:i + 1], streams=self.streams))

    def close(self) -> None:
        """Release the peer mappings (after the device has finished with them)."""
        torch.cuda.synchronize()
        for base in self._bases:
            check(lib().mr_ipc_close(base), "mr_ipc_close")
        self._bases = []
