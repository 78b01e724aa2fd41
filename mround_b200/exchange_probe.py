"""Time the weight-gradient exchange of one Qwen2.5-7B block across ranks.

Usage: python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1
       -m mround_b200.exchange_probe

For the block's four fused weight gradients (qkv, o, gate_up, down) at the
step's per-rank token count (16384 / N), four ways, each averaged over 10
iterations after 3 warm-up ones, CUDA events, max over ranks:

* ``gemm``: the four dW GEMMs only (no exchange -- the lower bound);
* ``nccl``: each dW GEMM into a local buffer, then an async NCCL
  reduce-scatter of its rows;
* ``p2p``: each dW GEMM storing its rows into the owners' slots over NVLink
  (``mr_gemm_rs``), then every owner's ordered sum (``mr_reduce_slots``);
* ``copy``: each dW GEMM into a local buffer, then the copy engines move each
  owner's rows into its slot (``mr_peer_send``), then the same ordered sum.

Rank 0 prints one line per way.
"""

from __future__ import annotations

import torch
import torch.distributed as tdist

from mround_b200 import kernels
from mround_b200.pipeline.dist import init_from_env
from mround_b200.pipeline.peer import PeerExchange

HIDDEN, KV, INTER, TOKENS = 3584, 512, 18944, 16384
SHAPES = [(HIDDEN + 2 * KV, HIDDEN), (HIDDEN, HIDDEN), (2 * INTER, HIDDEN), (HIDDEN, INTER)]


def main() -> None:
    dist = init_from_env("nccl", timeout_s=120.0)
    world, rank = dist.world, dist.rank
    dev = torch.device("cuda", torch.cuda.current_device())
    t = TOKENS // world
    gen = torch.Generator(device=dev).manual_seed(rank)
    ins = []
    for rows, cols in SHAPES:
        dy = kernels.split_bf16(torch.randn(t, rows, device=dev, generator=gen))
        x = kernels.split_bf16(torch.randn(t, cols, device=dev, generator=gen))
        ins.append((dy, x))
    grads = [torch.empty(r, c, device=dev) for r, c in SHAPES]
    shards = [torch.empty(r // world, c, device=dev) for r, c in SHAPES]
    peer = PeerExchange(dist, SHAPES, dev) if world > 1 else None
    copier = PeerExchange(dist, SHAPES, dev, copy_engine=True) if world > 1 else None
    epoch = 0

    def step(way: str) -> None:
        nonlocal epoch
        if way == "p2p":
            epoch += 1
            for (rows, cols), (dy, x), ex in zip(SHAPES, ins, peer.layers):
                kernels.gemm_rs(dy[0], dy[1], x[0], x[1], m=rows, n=cols, k=t, a_kmajor=False,
                                b_kmajor=False, lda=rows, ldb=cols, precision=3,
                                dst_ptrs=ex.dst_ptrs, ldd=cols, rows_per_rank=ex.rows_per_rank,
                                flag_ptrs=ex.flag_ptrs, done=ex.done, epoch=epoch)
            for ex, out in zip(peer.layers, shards):
                kernels.reduce_slots(ex.slots, ex.flags, epoch, out)
            return
        if way == "copy":
            epoch += 1
            for (rows, cols), (dy, x), g, ex in zip(SHAPES, ins, grads, copier.layers):
                kernels.gemm(dy[0], dy[1], x[0], x[1], g, m=rows, n=cols, k=t, a_kmajor=False,
                             b_kmajor=False, lda=rows, ldb=cols, ldc=cols, precision=3)
                ex.epoch = epoch
                ex.send(g)
            for ex in copier.layers:
                ex.wait_copies()
            for ex, out in zip(copier.layers, shards):
                kernels.reduce_slots(ex.slots, ex.flags, epoch, out)
            return
        works = []
        for (rows, cols), (dy, x), g, out in zip(SHAPES, ins, grads, shards):
            kernels.gemm(dy[0], dy[1], x[0], x[1], g, m=rows, n=cols, k=t, a_kmajor=False,
                         b_kmajor=False, lda=rows, ldb=cols, ldc=cols, precision=3)
            if way == "nccl" and world > 1:
                works.append(tdist.reduce_scatter_tensor(out, g, async_op=True))
        for w in works:
            w.wait()

    ways = ("gemm", "nccl", "p2p", "copy") if world > 1 else ("gemm",)
    for way in ways:
        for _ in range(3):
            step(way)
        dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(10):
            step(way)
        end.record()
        torch.cuda.synchronize()
        ms = dist.max_scalar(start.elapsed_time(end) / 10, dev)
        status = int(kernels.lib().mr_peer_status(1))
        if rank == 0:
            print(f"world {world} {way}: {ms:.3f} ms per block exchange (peer status {status})",
                  flush=True)
    dist.barrier()
    if peer is not None:
        peer.close()
        copier.close()
    if world > 1:
        tdist.destroy_process_group()


if __name__ == "__main__":
    main()
