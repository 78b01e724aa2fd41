"""Data-parallel step on 2 GPUs (NCCL) against one process on the whole batch.

Each rank holds half the sequences of the batch; the threshold comes from
all-reduced histograms, the weight gradients are reduce-scattered by rows --
by the weight-gradient GEMM itself storing rows into their owners' slots over
NVLink (or, for comparison, an NCCL reduce-scatter) -- each rank steps its rows
and the operands are all-gathered for the next step (two steps run).  Against a single-process step on the whole
batch: the loss agrees to float64 summation order and the exact outlier
threshold is identical; V after the steps agrees except where a gradient's
sign flips between two summation orders (bounded here at 0.1 % of entries);
and the two ranks hold bitwise identical parameters once gathered.  Skipped with fewer
than two GPUs.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ARCH = "tiny-qwen2"
SHAPE = (4, 64)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(device):
    from mround_b200.pipeline.arch import get_arch
    from mround_b200.pipeline.block import DeviceBlock
    from mround_b200.pipeline.model import SyntheticModel

    arch = get_arch(ARCH)
    params = SyntheticModel(arch, seed=21).block(0)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(*SHAPE, arch.hidden, generator=g) * 0.02
    tgt = x + 1e-3 * torch.randn(*SHAPE, arch.hidden, generator=g)
    return arch, DeviceBlock(arch, params, device), x, tgt


def _precision(name):
    from mround_b200.pipeline.block import TUNING_PRECISION, Precision

    return Precision() if name == "bf16x3" else TUNING_PRECISION


def _tuner(block, dist, exchange="p2p", prec="bf16x3", gather="codes"):
    from mround_b200.pipeline.tuning import BlockTuner
    from mround_b200.schemes import QuantScheme
    from oracle.block_tuner import LINEARS

    scheme = QuantScheme(bits=2, group_size=32, symmetry="asym")
    return BlockTuner(block, {p: scheme for p in LINEARS}, {p: 0.05 for p in LINEARS},
                      suppress=True, eps=1e-8, precision=_precision(prec), dist=dist,
                      exchange=exchange, gather=gather)


def _rank(rank, world, port, q, exchange="p2p", prec="bf16x3", gather="codes"):
    import torch.distributed as tdist

    from mround_b200.pipeline.dist import DistContext

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime

    tdist.init_process_group("nccl", rank=rank, world_size=world,
                             timeout=datetime.timedelta(seconds=120))
    try:
        ctx = DistContext(rank, world)
        dev = torch.device("cuda", rank)
        _, block, x, tgt = _setup(dev)
        rows = ctx.shard(SHAPE[0])
        tuner = _tuner(block, ctx, exchange, prec, gather)
        assert tuner.sharded, "tiny-qwen2's fused rows divide by 2: the row-sharded update runs"
        assert (tuner.peer is not None) == (exchange in ("p2p", "copy"))
        loss = tuner.step(x[rows].to(dev), tgt[rows].to(dev), 0, 10)
        # a second step runs on the all-gathered operands of the first
        loss2 = tuner.step(x[rows].to(dev), tgt[rows].to(dev), 1, 10)
        tuner.sync_params()
        total = torch.stack([loss, loss2])
        ctx.all_reduce_(total)
        torch.cuda.synchronize(dev)
        operands = [x.view(torch.int16).cpu().numpy() if x.dtype == torch.bfloat16
                    else x.cpu().numpy()
                    for t in tuner.tunables
                    for x in (t.layer.wq_hi, t.layer.wq_lo, t.layer.wq_t32) if x is not None]
        q.put((rank, total.tolist(), float(tuner.ws.thr.item()),
               [t.v.cpu().numpy() for t in tuner.tunables],
               [t.alpha.cpu().numpy() for t in tuner.tunables], operands))
        tuner.close()
        tdist.barrier()
    finally:
        tdist.destroy_process_group()


def _run_ranks(exchange, prec="bf16x3", gather="codes"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, exchange, prec, gather))
             for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("prec", ["bf16x3", "tuning"])
def test_two_gpu_fused_exchange_equals_nccl_reduce_scatter(prec):
    """The weight-gradient GEMM storing rows into their owners' slots over NVLink
    gives the same parameters, bit for bit, as the GEMM plus an NCCL
    reduce-scatter (two summands: the order cannot differ) -- with the bf16
    split and with the tuning default's tf32 products (mr_gemm_rs_tf32)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    fused = _run_ranks("p2p", prec)
    nccl = _run_ranks("nccl", prec)
    for a, b in zip(fused, nccl):
        assert a[1] == b[1] and a[2] == b[2]
        for x, y in zip(a[3] + a[4], b[3] + b[4]):
            assert np.array_equal(x, y)


@pytest.mark.parametrize("prec", ["bf16x3", "tuning"])
def test_two_gpu_codes_gather_equals_operands_gather(prec):
    """Gathering each rank's codes and per-group scale / zero point and
    rebuilding the operands on every rank gives the same operands, losses
    and parameters, bit for bit, as gathering the operands themselves."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    codes = _run_ranks("p2p", prec, "codes")
    operands = _run_ranks("p2p", prec, "operands")
    for a, b in zip(codes, operands):
        assert a[1] == b[1] and a[2] == b[2]
        assert len(a[5]) == len(b[5]) > 0
        for x, y in zip(a[3] + a[4] + a[5], b[3] + b[4] + b[5]):
            assert np.array_equal(x, y)


def test_two_gpu_copy_engine_exchange_equals_nccl_reduce_scatter():
    """The copy-engine form (local GEMM, cudaMemcpyAsync of each owner's rows
    into its slot, flag released after the copy) gives the same parameters,
    bit for bit, as the NCCL reduce-scatter."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    copied = _run_ranks("copy")
    nccl = _run_ranks("nccl")
    for a, b in zip(copied, nccl):
        assert a[1] == b[1] and a[2] == b[2]
        for x, y in zip(a[3] + a[4], b[3] + b[4]):
            assert np.array_equal(x, y)


@pytest.mark.parametrize("prec", ["bf16x3", "tuning"])
def test_two_gpu_step_matches_single_process(prec):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from mround_b200.pipeline.dist import DistContext

    res = _run_ranks("p2p", prec)
    # single process, whole batch, on GPU 0
    dev = torch.device("cuda", 0)
    _, block, x, tgt = _setup(dev)
    tuner = _tuner(block, DistContext(), prec=prec)
    loss = tuner.step(x.to(dev), tgt.to(dev), 0, 10)
    loss2 = tuner.step(x.to(dev), tgt.to(dev), 1, 10)
    torch.cuda.synchronize(dev)
    want_v = [t.v.cpu().numpy() for t in tuner.tunables]
    assert res[0][1][0] == pytest.approx(loss.item(), rel=1e-6)
    assert res[0][1][1] == pytest.approx(loss2.item(), rel=1e-4)
    assert res[0][2] == tuner.ws.thr.item()
    for a, b in zip(res[0][3], res[1][3]):
        assert np.array_equal(a, b), "ranks must hold identical parameters"
    for a, b in zip(res[0][4], res[1][4]):
        assert np.array_equal(a, b)
    differing = sum(int((a != b).sum()) for a, b in zip(res[0][3], want_v))
    total = sum(a.size for a in want_v)
    assert differing / total < 1e-3, f"{differing} of {total} V entries differ"


def _score_rank(rank, world, port, q):
    import datetime

    import torch.distributed as tdist

    from mround_b200.pipeline.dist import DistContext

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    tdist.init_process_group("nccl", rank=rank, world_size=world,
                             timeout=datetime.timedelta(seconds=120))
    try:
        got = _scores(torch.device("cuda", rank), DistContext(rank, world))
        q.put((rank, got))
        tdist.barrier()
    finally:
        tdist.destroy_process_group()


def _scores(device, dist):
    from mround_b200.pipeline.arch import get_arch
    from mround_b200.pipeline.model import SyntheticModel, zipf_tokens
    from mround_b200.pipeline.scoring import score_widths
    from mround_b200.schemes import QuantScheme

    model = SyntheticModel(get_arch(ARCH), seed=4)
    tokens = zipf_tokens(model.arch.vocab, 4, 33, seed=1)
    batches = [tokens[i:i + 1] for i in range(4)]
    scheme = QuantScheme(bits=4, group_size=32, symmetry="asym")
    return score_widths(model, batches, (2, 3, 4), scheme, device=device, dist=dist).scores


def test_two_gpu_scoring_matches_single_process():
    """DeltaLoss scoring with the batches split over two ranks (float64 sums
    all-reduced) equals the single-process scores, on both ranks."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from mround_b200.pipeline.dist import DistContext

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_score_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    want = _scores(torch.device("cuda", 0), DistContext())
    for _, got in res:
        assert set(got) == set(want)
        for layer in want:
            for bits in (2, 3, 4):
                assert got[layer][bits] == pytest.approx(want[layer][bits], rel=1e-12)
