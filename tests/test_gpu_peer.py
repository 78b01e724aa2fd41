"""The fused GEMM -> reduce-scatter pieces on one GPU: the remote epilogue of
K3 (``mr_gemm_rs``) with a single rank stores exactly what ``mr_gemm`` writes
and publishes its epoch; the owner-side sum (``mr_reduce_slots``) sums slots
in rank order; and a flag that nothing sets makes the bounded wait give up
with a status the host reads (no fault, the context stays usable)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200 import kernels

    return kernels


@pytest.mark.parametrize("m,n,k", [(512, 768, 1024), (4608 // 8 * 1, 3584 // 4, 2048)])
def test_gemm_rs_single_rank_equals_gemm(K, m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m + n)
    dy = torch.randn(k, m, device="cuda", generator=g)  # (tokens, out): MN-major A
    x = torch.randn(k, n, device="cuda", generator=g)   # (tokens, in): MN-major B
    a = K.split_bf16(dy)
    b = K.split_bf16(x)
    want = torch.empty(m, n, device="cuda")
    K.gemm(a[0], a[1], b[0], b[1], want, m=m, n=n, k=k, a_kmajor=False, b_kmajor=False, lda=m,
           ldb=n, ldc=n, precision=3)
    slot = torch.zeros(m, n, device="cuda")
    flags = torch.zeros(1, dtype=torch.int64, device="cuda")
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    for epoch in (1, 2):
        K.gemm_rs(a[0], a[1], b[0], b[1], m=m, n=n, k=k, a_kmajor=False, b_kmajor=False, lda=m,
                  ldb=n, precision=3, dst_ptrs=[slot.data_ptr()], ldd=n, rows_per_rank=m,
                  flag_ptrs=[flags.data_ptr()], done=done, epoch=epoch)
        torch.cuda.synchronize()
        assert torch.equal(slot, want)
        assert int(flags.item()) == epoch and int(done.item()) == 0
    out = torch.empty(m, n, device="cuda")
    K.reduce_slots(slot.view(1, m, n), flags, 2, out)
    torch.cuda.synchronize()
    assert torch.equal(out, want)


def test_gemm_rs_tf32_two_owners_equals_gemm(K):
    """The tf32 remote epilogue with 256-row tiles (two 128-row MMAs per K
    step): rows split between two owners (local buffers standing in for two
    ranks' slots; 2240 rows each, so a tile straddles the owners) hold
    exactly what mr_gemm_tf32 writes, and both flags carry the epoch."""
    m, n, k = 4480, 3584, 4096
    assert K.gemm_tile(m=m, n=n, k=k, precision=4, a_kmajor=False, b_kmajor=False)[0] == 256
    g = torch.Generator(device="cuda").manual_seed(3)
    dy = K.round_tf32(torch.randn(k, m, device="cuda", generator=g))  # MN-major A
    x = K.round_tf32(torch.randn(k, n, device="cuda", generator=g) * 0.02)  # MN-major B
    want = torch.empty(m, n, device="cuda")
    K.gemm_tf32(dy, x, want, m=m, n=n, k=k, a_kmajor=False, b_kmajor=False, lda=m, ldb=n, ldc=n)
    slots = torch.zeros(2, m // 2, n, device="cuda")
    flags = torch.zeros(2, dtype=torch.int64, device="cuda")
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.gemm_rs_tf32(dy, x, m=m, n=n, k=k, a_kmajor=False, b_kmajor=False, lda=m, ldb=n,
                   dst_ptrs=[slots[0].data_ptr(), slots[1].data_ptr()], ldd=n,
                   rows_per_rank=m // 2, flag_ptrs=[flags[0].data_ptr(), flags[1].data_ptr()],
                   done=done, epoch=5)
    torch.cuda.synchronize()
    assert torch.equal(slots.view(m, n), want)
    assert flags.tolist() == [5, 5] and int(done.item()) == 0


def test_reduce_slots_sums_in_rank_order(K):
    world, rows, cols = 4, 64, 96
    slots = torch.randn(world, rows, cols, device="cuda")
    flags = torch.full((world,), 5, dtype=torch.int64, device="cuda")
    out = torch.empty(rows, cols, device="cuda")
    K.reduce_slots(slots, flags, 5, out)
    torch.cuda.synchronize()
    want = ((slots[0] + slots[1]) + slots[2]) + slots[3]
    assert torch.equal(out, want)


def test_reduce_slots_wait_gives_up_with_a_status(K):
    from mround_b200._native import lib

    assert lib().mr_peer_status(1) == 0
    slots = torch.randn(2, 8, 16, device="cuda")
    flags = torch.tensor([3, 0], dtype=torch.int64, device="cuda")  # rank 1 never publishes
    out = torch.full((8, 16), 7.0, device="cuda")
    K.reduce_slots(slots, flags, 3, out)
    torch.cuda.synchronize()
    assert lib().mr_peer_status(1) == -5  # MR_ERR_TIMEOUT, cleared by the read
    assert torch.equal(out, torch.full((8, 16), 7.0, device="cuda")), "no partial sum is written"
    assert lib().mr_peer_status(0) == 0
    # the context is still usable
    assert float((slots.sum() - slots.sum()).item()) == 0.0
