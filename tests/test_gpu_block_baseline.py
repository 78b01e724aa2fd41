"""Block-level parity at the benchmark architectures, on the device.

The reference's bar (tests/unit/test_mlx_parity.py:95-98 of the reference):
one tuning step's loss and every V/alpha/beta gradient within 1e-3 relative
(max-normalised) of the float32 path, and a tuned block's final loss within
2 % of the float32 loop's (mround/pipeline/runner.py:790-953).  The
tiny-architecture tests in test_gpu_block.py check the same bars at hidden
128; these run them at the shapes the benchmark configurations name:

- SmolLM2-135M (hidden 576, 9/3 heads, SwiGLU 1536), W4 asym g64, 2 x 512
  tokens (configuration 1);
- Qwen2.5-0.5B (hidden 896, 14/2 heads, SwiGLU 4864, QKV bias), W2 asym g64,
  one 2048-token sequence (configuration 3);
- Qwen2.5-7B (hidden 3584, 28/4 heads -- GQA ratio 7 --, SwiGLU 18944), W2
  asym g64, one 2048-token sequence (configuration 5);

- Qwen2.5-3B (hidden 2048, 16/2 heads, SwiGLU 11008, QKV bias) under a mixed
  {2,3,4}-bit symmetric plan with searched scales, one 2048-token sequence
  (configuration 4's scheme at its architecture);

and a tuning loop at configuration 1 (SmolLM2, 50 steps, 4 x 8 x 512 tokens).

Sequences of 512 and 2048 tokens take the causal tile-skipping GEMM modes and
the band-limited softmax, which the hidden-128 tests at 64 tokens do not.
Inputs are block-0 inputs of the benchmark's kind (token embeddings,
N(0, 0.02)); V/alpha/beta are perturbed away from their initial values so
that every gradient term is exercised.  The device side runs through the C
ABI (``BlockTuner`` on ``libmround_b200.so``); the oracle is the torch-CPU
float32 restatement in ``oracle/block_tuner.py``.
"""

from __future__ import annotations

import time

import pytest
import torch

from oracle.block_tuner import LINEARS, OracleBlock, loss_fn, tune_block
from tests.conftest import relative_error

pytestmark = pytest.mark.gpu

GROUP = 64
# name -> (bits, suppress outliers, sequences, tokens per sequence)
STEP_CASES = {
    "smollm2-135m": (4, False, 2, 512),
    "qwen2.5-0.5b": (2, True, 1, 2048),
    "qwen2.5-7b": (2, True, 1, 2048),
}


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200.pipeline import arch as A
    from mround_b200.pipeline.model import SyntheticModel

    return A, SyntheticModel


def block_inputs(arch, n_batches, bsz, seq, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(bsz, seq, arch.hidden, generator=g) * 0.02 for _ in range(n_batches)]


def perturbed(oracle, seed):
    g = torch.Generator().manual_seed(seed)
    out = {}
    for p in LINEARS:
        v, a, b = oracle.init_params()[p]
        out[p] = ((torch.rand(v.shape, generator=g) - 0.5) * 0.6,
                  0.7 + 0.3 * torch.rand(a.shape, generator=g),
                  0.7 + 0.3 * torch.rand(b.shape, generator=g))
    return out


@pytest.mark.parametrize("prec_name", ["bf16x3", "tuning"])
@pytest.mark.parametrize("name", list(STEP_CASES))
def test_step_matches_oracle_at_benchmark_shape(env, name, prec_name):
    """One step's loss and V/alpha/beta gradients against the oracle.

    The outlier rule makes dL/dpred a discontinuous function of the residual:
    an element whose |r| lies within the implementations' rounding difference
    of the k-th largest can be excluded by one and kept by the other, and at
    the 7B shape one such element moves a gradient row by a few percent.  The
    kernels cannot agree on those elements unless they round identically (the
    reference's own MLX path differs from its NumPy oracle by 8.5e-4 in every
    matmul).  So the check is split: the loss, the selected threshold and the
    outlier sets are compared directly (the sets may differ in a handful of
    boundary elements), and the gradients are compared at the oracle's
    outlier set -- the smooth part, where the 1e-3 bar is meaningful.  The
    gradients at each side's own set are printed, not asserted."""
    A, SM = env
    from mround_b200.pipeline.block import TUNING_PRECISION, DeviceBlock, Precision
    from mround_b200.pipeline.dist import DistContext
    from mround_b200.pipeline.tuning import BlockTuner
    from mround_b200.schemes import QuantScheme

    # three bf16 products in every GEMM, or the tuning default (tf32 backward)
    prec = Precision() if prec_name == "bf16x3" else TUNING_PRECISION
    bits, suppress, bsz, seq = STEP_CASES[name]
    arch = A.get_arch(name)
    params = SM(arch, seed=5).block(0)
    oracle = OracleBlock(arch, params, {p: bits for p in LINEARS}, GROUP)
    x = block_inputs(arch, 1, bsz, seq, seed=1)[0]
    t0 = time.perf_counter()
    with torch.no_grad():
        target = oracle.forward(x)
    qp = perturbed(oracle, seed=9)
    leaves = {p: tuple(t.clone().requires_grad_(True) for t in qp[p]) for p in LINEARS}
    pred_o = oracle.forward(x, leaves)
    loss_o, thr_o = loss_fn(pred_o, target, suppress)
    loss_o.backward()
    t_oracle = time.perf_counter() - t0
    r_o = (pred_o.detach() - target).abs()
    n = r_o.numel()
    keep_o = r_o < thr_o if suppress else torch.ones_like(r_o, dtype=torch.bool)

    scheme = QuantScheme(bits=bits, group_size=GROUP, symmetry="asym")
    block = DeviceBlock(arch, params)
    tuner = BlockTuner(block, {p: scheme for p in LINEARS}, {p: 0.01 for p in LINEARS},
                       suppress=suppress, eps=1e-8, precision=prec, dist=DistContext())
    for t in tuner.tunables:
        for m in t.members:
            v, a, b = qp[m.path]
            t.load(m.path, v.cuda(), a.cuda(), b.cuda())
    xd, td = x.cuda(), target.cuda()

    def grad_errors(grads):
        worst = {}
        for p in LINEARS:
            for i, nm in enumerate(("v", "alpha", "beta")):
                worst[f"{p}.{nm}"] = relative_error(grads[p][i].cpu().numpy(),
                                                    leaves[p][i].grad.numpy())
        return worst

    # the device's own step: K4's loss, threshold and outlier set
    loss_d, grads_own = tuner.gradient_only(xd, td)
    torch.cuda.synchronize()
    loss_err = abs(loss_d.item() - loss_o.item()) / loss_o.item()
    own = grad_errors(grads_own)
    # the same step at the oracle's outlier set (dL/dpred formed from it)
    with torch.no_grad():
        out, saved = block.forward_fused(xd, prec, True)
        r_d = out - td
        keep = keep_o.cuda()
        grad = (2.0 * r_d * keep / n).float().contiguous()
        block.backward_fused(saved, grad, prec)
        del saved
    grads = {}
    for t in tuner.tunables:
        grads.update(t.gradients())
    torch.cuda.synchronize()
    common = grad_errors(grads)
    top = max(common, key=common.__getitem__)
    top_own = max(own, key=own.__getitem__)
    flips = int(((r_d.abs().cpu() < thr_o) != keep_o).sum()) if suppress else 0
    thr_note = ""
    if suppress:
        thr_d = float(tuner.ws.thr.item())
        thr_err = abs(thr_d - float(thr_o)) / float(thr_o)
        thr_note = f", threshold rel {thr_err:.1e}, {flips} of {n} elements on the other side"
    print(f"[block parity] {name} {prec_name} W{bits} g{GROUP} {bsz}x{seq}: loss rel "
          f"{loss_err:.2e}{thr_note}; "
          f"worst gradient {common[top]:.2e} ({top}) at the oracle's outlier set, "
          f"{own[top_own]:.2e} ({top_own}) at its own; oracle {t_oracle:.1f} s")
    assert loss_err <= 1e-3
    assert common[top] < 1e-3, common
    if suppress:
        assert thr_err < 1e-4
        # boundary elements only: at most 0.5 % of the k excluded ones
        k = max(1, int(n * 0.001))
        assert flips <= max(4, k // 200), flips
    else:
        assert own[top_own] < 1e-3, own


# name -> (bits, suppress outliers, batches, sequences per batch, tokens, iters)
LOOP_CASES = {
    # configuration 1 at the block level: W4 g64, 32 x 512 tokens in batches
    # of 8, 50 steps at lr 1/50, no outlier suppression (4 bits)
    "smollm2-135m": (4, False, 4, 8, 512, 50),
}
# No short loop runs at the 7B shape: a 20-step loop at lr 1/20 over two
# one-sequence batches is chaotic in the rounding -- across input seeds the
# float32 oracle and the bf16x3 device path end -5.8 %, +2.6 % and +5.8 %
# apart, and with the outlier rule on, the oracle in float64 ends 25 % away
# from itself in float32 -- so a 2 % bar there would test the noise.  The 7B
# shape is covered by the step test above; whole-recipe loops (200 steps,
# 8 x 2048 batches) are compared outside the test suite.


@pytest.mark.parametrize("name", list(LOOP_CASES))
def test_tuning_loop_matches_oracle_at_benchmark_shape(env, name):
    """The runner's default tuning step (tf32 backward products) over a whole
    loop: initial loss within 1e-3 and final loss within 2 % of the oracle's."""
    A, SM = env
    from mround_b200.pipeline.block import DeviceBlock
    from mround_b200.pipeline.runner import QuantizationRunner
    from mround_b200.schemes import QuantScheme, TuningConfig

    bits, suppress, n_batches, bsz, seq, iters = LOOP_CASES[name]
    arch = A.get_arch(name)
    params = SM(arch, seed=11).block(0)
    oracle = OracleBlock(arch, params, {p: bits for p in LINEARS}, GROUP)
    inputs = block_inputs(arch, n_batches, bsz, seq, seed=2)
    t0 = time.perf_counter()
    with torch.no_grad():
        targets = [oracle.forward(x) for x in inputs]
    ref = tune_block(oracle, inputs, targets, iters=iters, lr0=1.0 / iters, suppress=suppress)
    t_oracle = time.perf_counter() - t0

    scheme = QuantScheme(bits=bits, group_size=GROUP, symmetry="asym")
    tuning = TuningConfig(iters=iters, batch_size=bsz, n_samples=n_batches * bsz, seq_len=seq,
                          suppress_outliers=suppress)
    runner = QuantizationRunner(scheme, tuning)
    block = DeviceBlock(arch, params)
    result, _ = runner.quantize_block(block, "model.layers.0", [x.cuda() for x in inputs],
                                      [t.cuda() for t in targets])
    init_err = abs(result.initial_loss - ref["initial_loss"]) / ref["initial_loss"]
    final_err = abs(result.final_loss - ref["final_loss"]) / ref["final_loss"]
    print(f"[loop parity] {name} W{bits} g{GROUP} {n_batches}x{bsz}x{seq}, {iters} steps: "
          f"initial rel {init_err:.2e}, final {result.final_loss:.5e} vs oracle "
          f"{ref['final_loss']:.5e} (rel {final_err:.2e}); oracle {t_oracle:.1f} s")
    assert init_err <= 1e-3
    assert final_err <= 0.02
    assert result.final_loss < result.initial_loss
    assert not ref["reverted"]


# configuration 4's scheme at its architecture: Qwen2.5-3B (hidden 2048, 16/2
# heads, SwiGLU 11008, QKV bias), symmetric with the searched scale, a mixed
# plan over {2, 3, 4} bits (widths differ inside the fused qkv and gate_up)
MIXED_BITS = {"self_attn.q_proj": 4, "self_attn.k_proj": 3, "self_attn.v_proj": 3,
              "self_attn.o_proj": 2, "mlp.gate_proj": 3, "mlp.up_proj": 2, "mlp.down_proj": 4}


def test_mixed_searched_step_matches_oracle_at_3b_shape(env):
    """One tuning step (the runner's default precision) of a 3B block under a
    mixed {2,3,4}-bit symmetric plan with searched scales: the device's
    searched scales feed the oracle, then loss and V/beta gradients at the
    oracle's outlier set within 1e-3 (alpha is inert under a searched scale)."""
    A, SM = env
    from mround_b200.pipeline.block import TUNING_PRECISION, DeviceBlock
    from mround_b200.pipeline.dist import DistContext
    from mround_b200.pipeline.tuning import BlockTuner
    from mround_b200.schemes import QuantScheme

    arch = A.get_arch("qwen2.5-3b")
    params = SM(arch, seed=8).block(0)
    x = block_inputs(arch, 1, 1, 2048, seed=4)[0]
    schemes = {p: QuantScheme(bits=b, group_size=GROUP, symmetry="sym", scale_init="searched")
               for p, b in MIXED_BITS.items()}
    block = DeviceBlock(arch, params)
    tuner = BlockTuner(block, schemes, {p: 0.01 for p in LINEARS}, suppress=True, eps=1e-8,
                       precision=TUNING_PRECISION, dist=DistContext())
    assert tuner.search([x.cuda()]) > 0.0
    init = {}
    for t in tuner.tunables:
        for m in t.members:
            r0, r1 = m.rows
            init[m.path] = t.init_scale[r0:r1].cpu()
    oracle = OracleBlock(arch, params, MIXED_BITS, GROUP, symmetric=True, init_scales=init)
    with torch.no_grad():
        target = OracleBlock(arch, params, MIXED_BITS, GROUP).forward(x)
    g = torch.Generator().manual_seed(12)
    qp = {}
    for p in LINEARS:
        v, a, b = oracle.init_params()[p]
        qp[p] = ((torch.rand(v.shape, generator=g) - 0.5) * 0.6,
                 0.5 + torch.rand(a.shape, generator=g),
                 0.5 + torch.rand(b.shape, generator=g))
    leaves = {p: tuple(t.clone().requires_grad_(True) for t in qp[p]) for p in LINEARS}
    pred_o = oracle.forward(x, leaves)
    loss_o, thr_o = loss_fn(pred_o, target, True)
    loss_o.backward()
    keep_o = (pred_o.detach() - target).abs() < thr_o
    n = keep_o.numel()
    for t in tuner.tunables:
        for m in t.members:
            v, a, b = qp[m.path]
            t.load(m.path, v.cuda(), a.cuda(), b.cuda())
    loss_d, _ = tuner.gradient_only(x.cuda(), target.cuda())
    with torch.no_grad():
        out, saved = block.forward_fused(x.cuda(), TUNING_PRECISION, True)
        r_d = out - target.cuda()
        grad = (2.0 * r_d * keep_o.cuda() / n).float().contiguous()
        block.backward_fused(saved, grad, TUNING_PRECISION)
        del saved
    grads = {}
    for t in tuner.tunables:
        grads.update(t.gradients())
    torch.cuda.synchronize()
    loss_err = abs(loss_d.item() - loss_o.item()) / loss_o.item()
    worst = {}
    for p in LINEARS:
        for i, nm in ((0, "v"), (2, "beta")):
            worst[f"{p}.{nm}"] = relative_error(grads[p][i].cpu().numpy(),
                                                leaves[p][i].grad.numpy())
        assert not grads[p][1].any(), "alpha is inert under a searched scale"
    top = max(worst, key=worst.__getitem__)
    thr_err = abs(float(tuner.ws.thr.item()) - float(thr_o)) / float(thr_o)
    print(f"[block parity] qwen2.5-3b mixed {{2,3,4}} sym searched g{GROUP} 1x2048: loss rel "
          f"{loss_err:.2e}, threshold rel {thr_err:.1e}; worst gradient {worst[top]:.2e} ({top})")
    assert loss_err <= 1e-3
    assert thr_err < 1e-4
    assert worst[top] < 1e-3, worst
