"""Block-level parity: the device tuning step against the torch-CPU float32 oracle.

Bars (from the reference's parity suite and the run's target): per-step loss
and parameter gradients within 1e-3 relative (max-normalised,
tests/unit/test_mlx_parity.py:95-98) of the float32 path; the tuned block's
final loss within 2 % of the oracle's; block outputs (targets) to float32
precision.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.block_tuner import LINEARS, OracleBlock, loss_fn, tune_block
from tests.conftest import relative_error

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200.pipeline import arch as A
    from mround_b200.pipeline.model import SyntheticModel

    return A, SyntheticModel


def make_inputs(arch, n_batches, bsz, seq, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(bsz, seq, arch.hidden, generator=g) * 0.02 for _ in range(n_batches)]


@pytest.mark.parametrize("name", ["tiny-qwen2", "tiny-llama"])
def test_dense_forward_matches_oracle(env, name):
    A, SM = env
    from mround_b200.pipeline.block import DeviceBlock, Precision

    arch = A.get_arch(name)
    params = SM(arch, seed=3).block(0)
    x = make_inputs(arch, 1, 2, 64)[0]
    want = OracleBlock(arch, params, {p: 4 for p in LINEARS}, 32).forward(x)
    with torch.no_grad():
        got = DeviceBlock(arch, params).forward(x.cuda(), Precision()).cpu()
    assert relative_error(got.numpy(), want.numpy()) < 2e-5


def perturbed(oracle, seed):
    g = torch.Generator().manual_seed(seed)
    out = {}
    for p in LINEARS:
        v, a, b = oracle.init_params()[p]
        out[p] = ((torch.rand(v.shape, generator=g) - 0.5) * 0.6,
                  0.7 + 0.3 * torch.rand(a.shape, generator=g),
                  0.7 + 0.3 * torch.rand(b.shape, generator=g))
    return out


@pytest.mark.parametrize("bits,suppress", [(2, True), (4, False)])
@pytest.mark.parametrize("prec", [(3, 3, 3)])
def test_step_loss_and_gradients_match_oracle(env, bits, suppress, prec):
    A, SM = env
    from mround_b200.pipeline.block import DeviceBlock, Precision
    from mround_b200.pipeline.dist import DistContext
    from mround_b200.pipeline.tuning import BlockTuner
    from mround_b200.schemes import QuantScheme

    arch = A.get_arch("tiny-qwen2")
    params = SM(arch, seed=5).block(0)
    group = 32
    oracle = OracleBlock(arch, params, {p: bits for p in LINEARS}, group)
    x = make_inputs(arch, 1, 2, 64, seed=1)[0]
    with torch.no_grad():
        target = oracle.forward(x)
    qp = perturbed(oracle, seed=9)
    leaves = {p: tuple(t.clone().requires_grad_(True) for t in qp[p]) for p in LINEARS}
    loss_o, _ = loss_fn(oracle.forward(x, leaves), target, suppress)
    loss_o.backward()

    scheme = QuantScheme(bits=bits, group_size=group, symmetry="asym")
    block = DeviceBlock(arch, params)
    tuner = BlockTuner(block, {p: scheme for p in LINEARS}, {p: 0.01 for p in LINEARS},
                       suppress=suppress, eps=1e-8, precision=Precision(*prec), dist=DistContext())
    for t in tuner.tunables:
        for m in t.members:
            v, a, b = qp[m.path]
            t.load(m.path, v.cuda(), a.cuda(), b.cuda())
    loss_d, grads = tuner.gradient_only(x.cuda(), target.cuda())
    torch.cuda.synchronize()
    assert abs(loss_d.item() - loss_o.item()) <= 1e-3 * loss_o.item()
    worst = {}
    for p in LINEARS:
        for i, nm in enumerate(("v", "alpha", "beta")):
            got = grads[p][i].cpu().numpy()
            want = leaves[p][i].grad.numpy()
            worst[f"{p}.{nm}"] = relative_error(got, want)
    print("max-normalised gradient error", prec, max(worst.values()))
    assert max(worst.values()) < 1e-3, worst


def test_tuning_loop_matches_oracle(env):
    A, SM = env
    from mround_b200.pipeline.block import DeviceBlock, Precision
    from mround_b200.pipeline.runner import QuantizationRunner
    from mround_b200.schemes import QuantScheme, TuningConfig

    arch = A.get_arch("tiny-qwen2")
    params = SM(arch, seed=11).block(0)
    bits, group, iters = 2, 32, 20
    oracle = OracleBlock(arch, params, {p: bits for p in LINEARS}, group)
    inputs = make_inputs(arch, 4, 2, 64, seed=2)
    with torch.no_grad():
        targets = [oracle.forward(x) for x in inputs]
    ref = tune_block(oracle, inputs, targets, iters=iters, lr0=1.0 / iters, suppress=True)

    scheme = QuantScheme(bits=bits, group_size=group, symmetry="asym")
    tuning = TuningConfig(iters=iters, batch_size=2, n_samples=8, seq_len=64)
    runner = QuantizationRunner(scheme, tuning)
    block = DeviceBlock(arch, params)
    result, layers = runner.quantize_block(block, "model.layers.0", [x.cuda() for x in inputs],
                                           [t.cuda() for t in targets])
    assert result.initial_loss == pytest.approx(ref["initial_loss"], rel=1e-3)
    assert result.final_loss == pytest.approx(ref["final_loss"], rel=0.02)
    assert result.final_loss < result.initial_loss
    assert set(layers) == {f"model.layers.0.{p}" for p in LINEARS}


def test_advance_uses_bf16_reconstruction(env):
    """After commit the block runs on bf16(Wq), as the reference's committed layer does."""
    A, SM = env
    from mround_b200.pipeline.block import DeviceBlock, Precision
    from mround_b200.pipeline.dist import DistContext
    from mround_b200.pipeline.tuning import BlockTuner
    from mround_b200.schemes import QuantScheme
    from oracle import quant_fp32

    arch = A.get_arch("tiny-llama")
    params = SM(arch, seed=2).block(0)
    scheme = QuantScheme(bits=3, group_size=32, symmetry="asym")
    block = DeviceBlock(arch, params)
    tuner = BlockTuner(block, {p: scheme for p in LINEARS}, {p: 0.01 for p in LINEARS},
                       suppress=False, eps=1e-8, precision=Precision(), dist=DistContext())
    tuner.commit()
    committed = {}
    for p in LINEARS:
        w = params.linears[p].float().numpy()
        ones = np.ones((w.shape[0], w.shape[1] // 32), np.float32)
        qdq, _, _, _ = quant_fp32.fake_quantize(w, np.zeros_like(w), ones, ones, 3, 32)
        committed[p] = torch.from_numpy(qdq).to(torch.bfloat16).float()
    oracle = OracleBlock(arch, params, {p: 3 for p in LINEARS}, 32)
    oracle.committed = committed
    x = make_inputs(arch, 1, 2, 32, seed=4)[0]
    with torch.no_grad():
        got = block.forward(x.cuda(), Precision()).cpu()
    assert relative_error(got.numpy(), oracle.forward(x).numpy()) < 2e-5


@pytest.mark.parametrize("name,seq", [("tiny-qwen2", 64), ("tiny-llama", 64), ("tiny-qwen2", 256),
                                      ("tiny-llama", 384)])
def test_fused_path_matches_autograd_path(env, name, seq):
    """The explicit fused forward/backward equals the autograd composition of
    the same kernels: outputs and every fused weight gradient."""
    A, SM = env
    from mround_b200.pipeline.block import DeviceBlock, Precision
    from mround_b200.pipeline.dist import DistContext
    from mround_b200.pipeline.tuning import BlockTuner
    from mround_b200.schemes import QuantScheme

    arch = A.get_arch(name)
    params = SM(arch, seed=8).block(0)
    scheme = QuantScheme(bits=3, group_size=32, symmetry="asym")
    block = DeviceBlock(arch, params)
    tuner = BlockTuner(block, {p: scheme for p in LINEARS}, {p: 0.01 for p in LINEARS},
                       suppress=False, eps=1e-8, precision=Precision(), dist=DistContext())
    # seq % 128 == 0 exercises the causal tile-skipping GEMM modes and band softmax
    x = make_inputs(arch, 1, 2, seq, seed=5)[0].cuda()
    g = torch.randn(x.shape, device="cuda") * 1e-3
    xa = x.clone().requires_grad_(True)
    out_a = block.forward(xa, Precision(), train=True)
    out_a.backward(g)
    grads_a = {n: l.grad.clone() for n, l in block.layers.items()}
    out_f, saved = block.forward_fused(x, Precision(), True)
    dx = block.backward_fused(saved, g, Precision(), want_dx=True)
    torch.cuda.synchronize()
    assert relative_error(out_f.detach().cpu().numpy(), out_a.detach().cpu().numpy()) < 1e-5
    for n, l in block.layers.items():
        assert relative_error(l.grad.cpu().numpy(), grads_a[n].cpu().numpy()) < 1e-4, n
    # the block-input gradient (used by the scoring backward)
    assert relative_error(dx.cpu().numpy(), xa.grad.cpu().numpy()) < 1e-4
    del tuner
