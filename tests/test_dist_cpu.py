"""Data-parallel host logic on CPU ranks (gloo, world size 2).

- The exact global outlier threshold from per-rank radix histograms summed by
  an all-reduce equals the k-th largest |r| of the whole batch.
- Per-rank weight gradients summed by an all-reduce give every rank the same
  signed step, equal to the single-process step on the whole batch.
- Loss shares divided by the global element count sum to the batch loss.
- The row-sharded exchange (reduce-scatter of the gradient by rows, each rank
  stepping its own rows, all-gather of the result) equals the replicated step.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import losses_fp32 as L
from oracle import quant_fp32 as Q


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mround_b200.pipeline.dist import DistContext

        ctx = DistContext(rank, world)
        rng = np.random.default_rng(0)
        batch = rng.standard_t(3, size=(4, 64, 96)).astype(np.float32)  # all ranks see the seed
        shard = batch[ctx.shard(batch.shape[0])]
        # (1) threshold by summed histograms
        n_global = batch.size
        k = L.outlier_k(n_global)
        prefix, mask, k_left = 0, 0, k
        for p in range(3):
            h = torch.from_numpy(L.radix_digit_hist(shard, p, prefix, mask))
            ctx.all_reduce_(h)
            prefix, mask, k_left = L.radix_select_step(h.numpy(), k_left, p, prefix, mask)
        thr = np.uint32(prefix).view(np.float32)
        # (2) loss shares
        loss_share, _, _ = L.loss_and_grad(shard, np.zeros_like(shard), suppress=True,
                                           elements=n_global, threshold=thr)
        t = torch.tensor([loss_share], dtype=torch.float64)
        ctx.all_reduce_(t)
        # (3) gradient sum then identical step
        w = rng.normal(0, 0.02, size=(8, 64)).astype(np.float32)
        g_full = rng.normal(0, 1e-3, size=(4, 8, 64)).astype(np.float32)
        g_local = torch.from_numpy(g_full[ctx.shard(4)].sum(0))
        ctx.all_reduce_(g_local)
        ones = np.ones((8, 1), np.float32)
        gv, ga, gb = Q.ste_grads(w, np.zeros_like(w), ones, ones, g_local.numpy(), 2, 64)
        v1, a1, b1 = Q.signsgd_step(np.zeros_like(w), ones, ones, gv, ga, gb, 0.005, 0.1, 1.0)
        # (4) row-sharded: reduce-scatter rows, step own rows, all-gather V
        per = w.shape[0] // world
        r0, r1 = rank * per, (rank + 1) * per
        g_rows = torch.empty((per, w.shape[1]), dtype=torch.float32)
        work = ctx.reduce_scatter_async(g_rows, torch.from_numpy(np.ascontiguousarray(g_full[ctx.shard(4)].sum(0))))
        work.wait()
        o = ones[r0:r1]
        gvr, gar, gbr = Q.ste_grads(w[r0:r1], np.zeros_like(w[r0:r1]), o, o, g_rows.numpy(), 2, 64)
        vr, _, _ = Q.signsgd_step(np.zeros_like(w[r0:r1]), o, o, gvr, gar, gbr, 0.005, 0.1, 1.0)
        v_sharded = torch.empty(w.shape, dtype=torch.float32)
        ctx.all_gather_async(v_sharded, torch.from_numpy(np.ascontiguousarray(vr))).wait()
        q.put((rank, float(thr), float(t.item()), v1, a1, b1, v_sharded.numpy()))
    finally:
        dist.destroy_process_group()


def test_two_rank_exchange_matches_single_process():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort(key=lambda r: r[0])
    rng = np.random.default_rng(0)
    batch = rng.standard_t(3, size=(4, 64, 96)).astype(np.float32)
    want_thr = L.outlier_threshold(batch)
    want_loss, _, _ = L.loss_and_grad(batch, np.zeros_like(batch), suppress=True)
    w = rng.normal(0, 0.02, size=(8, 64)).astype(np.float32)
    g_full = rng.normal(0, 1e-3, size=(4, 8, 64)).astype(np.float32)
    ones = np.ones((8, 1), np.float32)
    gv, ga, gb = Q.ste_grads(w, np.zeros_like(w), ones, ones, g_full.sum(0), 2, 64)
    v_want, _, _ = Q.signsgd_step(np.zeros_like(w), ones, ones, gv, ga, gb, 0.005, 0.1, 1.0)
    for rank, thr, loss, v1, a1, b1, v_sharded in results:
        assert thr == want_thr, "histogram exchange gives the exact global order statistic"
        assert loss == pytest.approx(want_loss, rel=1e-12)
        assert np.array_equal(v1, v_want)
        assert np.array_equal(v_sharded, v_want), "row-sharded step equals the replicated one"
    assert np.array_equal(results[0][3], results[1][3])
    assert np.array_equal(results[0][4], results[1][4])


def test_shards_partition_the_batch():
    from mround_b200.pipeline.dist import DistContext

    for world in (1, 2, 4, 8):
        seen = sorted(j for r in range(world) for j in DistContext(r, world).shard(8))
        assert seen == list(range(8))
