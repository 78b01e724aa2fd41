"""Block-level parity of the symmetric and searched schemes: one step's loss
and gradients, the search stage (importance statistics and searched scales),
and a short tuning loop, against the torch-CPU float32 oracle.

Bars as for the asymmetric block tests: loss and gradients within 1e-3
max-normalised (tests/unit/test_mlx_parity.py:95-98), the tuned block's final
loss within 2 % of the oracle's.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import scale_search as o_s
from oracle.block_tuner import (LINEARS, OracleBlock, attention, loss_fn, rms_norm, rope,
                                tune_block)
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


def scheme_for(kind, bits, group):
    from mround_b200.schemes import QuantScheme

    init = "searched" if kind == "searched" else "observed_range"
    return QuantScheme(bits=bits, group_size=group, symmetry="sym", scale_init=init)


def tuner_for(block, scheme, suppress):
    from mround_b200.pipeline.block import Precision
    from mround_b200.pipeline.dist import DistContext
    from mround_b200.pipeline.tuning import BlockTuner

    return BlockTuner(block, {p: scheme for p in LINEARS}, {p: 0.01 for p in LINEARS},
                      suppress=suppress, eps=1e-8, precision=Precision(), dist=DistContext())


def device_init_scales(tuner):
    out = {}
    for t in tuner.tunables:
        for m in t.members:
            r0, r1 = m.rows
            out[m.path] = t.init_scale[r0:r1].cpu()
    return out


def oracle_importance(ob: OracleBlock, x):
    """Summed squared input of every linear under the dense block (float64)."""
    ar = ob.arch
    bsz, s, _ = x.shape
    seen = {}

    def lin(p, inp):
        key = {"self_attn.q_proj": "qkv", "self_attn.o_proj": "o", "mlp.gate_proj": "gate_up",
               "mlp.down_proj": "down"}.get(p)
        if key is not None:
            seen[key] = inp.reshape(-1, inp.shape[-1]).double().pow(2).sum(0)
        y = inp @ ob.w[p].t()
        return y + ob.b[p] if p in ob.b else y

    h1 = rms_norm(x, ob.n_in, ar.rms_eps)
    q = lin("self_attn.q_proj", h1).view(bsz, s, ar.heads, ar.head_dim).transpose(1, 2)
    k = lin("self_attn.k_proj", h1).view(bsz, s, ar.kv_heads, ar.head_dim).transpose(1, 2)
    v = lin("self_attn.v_proj", h1).view(bsz, s, ar.kv_heads, ar.head_dim).transpose(1, 2)
    q, k = rope(q, ar.rope_theta), rope(k, ar.rope_theta)
    att = attention(q, k, v, 1.0 / math.sqrt(ar.head_dim)).transpose(1, 2).reshape(bsz, s, -1)
    h = x + lin("self_attn.o_proj", att)
    h2 = rms_norm(h, ob.n_post, ar.rms_eps)
    lin("mlp.down_proj", F.silu(lin("mlp.gate_proj", h2)) * lin("mlp.up_proj", h2))
    return seen


@pytest.mark.parametrize("kind", ["sym", "searched"])
@pytest.mark.parametrize("bits,suppress", [(2, True), (4, False)])
def test_sym_step_loss_and_gradients_match_oracle(env, kind, bits, suppress):
    A, SM = env
    from mround_b200.pipeline.block import DeviceBlock

    arch = A.get_arch("tiny-qwen2")
    params = SM(arch, seed=5).block(0)
    group = 32
    x = make_inputs(arch, 1, 2, 64, seed=1)[0]
    block = DeviceBlock(arch, params)
    tuner = tuner_for(block, scheme_for(kind, bits, group), suppress)
    init = None
    if kind == "searched":
        assert tuner.search([x.cuda()]) > 0.0
        init = device_init_scales(tuner)
    oracle = OracleBlock(arch, params, {p: bits for p in LINEARS}, group, symmetric=True,
                         init_scales=init)
    with torch.no_grad():
        target = OracleBlock(arch, params, {p: bits for p in LINEARS}, group).forward(x)
    g = torch.Generator().manual_seed(9)
    lo, hi = (0.5, 1.5) if kind == "searched" else (0.7, 1.0)
    qp = {}
    for p in LINEARS:
        v, a, b = oracle.init_params()[p]
        qp[p] = ((torch.rand(v.shape, generator=g) - 0.5) * 0.6,
                 lo + (hi - lo) * torch.rand(a.shape, generator=g),
                 lo + (hi - lo) * torch.rand(b.shape, generator=g))
    leaves = {p: tuple(t.clone().requires_grad_(True) for t in qp[p]) for p in LINEARS}
    loss_o, _ = loss_fn(oracle.forward(x, leaves), target, suppress)
    loss_o.backward()
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
            leaf = leaves[p][i]
            # alpha does not enter a searched scale: autograd leaves it without a gradient
            want = leaf.grad.numpy() if leaf.grad is not None else np.zeros(tuple(leaf.shape), np.float32)
            got = grads[p][i].cpu().numpy()
            if not np.abs(want).max() and not np.abs(got).max():
                continue  # alpha under a searched scale: zero on both sides
            worst[f"{p}.{nm}"] = relative_error(got, want)
    assert max(worst.values()) < 1e-3, worst
    if kind == "searched":
        assert all(not grads[p][1].any() for p in LINEARS), "alpha is inert"


def test_search_stage_matches_oracle(env):
    A, SM = env
    from mround_b200.pipeline.block import DeviceBlock

    arch = A.get_arch("tiny-llama")
    params = SM(arch, seed=6).block(0)
    inputs = make_inputs(arch, 3, 2, 64, seed=3)
    block = DeviceBlock(arch, params)
    tuner = tuner_for(block, scheme_for("searched", 2, 32), True)
    tuner.search([x.cuda() for x in inputs])
    torch.cuda.synchronize()
    ob = OracleBlock(arch, params, {p: 2 for p in LINEARS}, 32)
    want = {}
    with torch.no_grad():
        for x in inputs:
            for k, v in oracle_importance(ob, x).items():
                want[k] = want.get(k, 0) + v
    for name, got in tuner.importance.items():
        assert relative_error(got.cpu().numpy(), want[name].numpy()) < 1e-4, name
    # the searched scales are the search of the device's importance, exactly,
    # and operands were formed from them
    for t in tuner.tunables:
        imp = tuner.importance[t.layer.name].cpu().numpy()
        for m in t.members:
            r0, r1 = m.rows
            w = params.linears[m.path].float().numpy()
            expect = o_s.search_scales_f32(w, 2, 32, imp).reshape(r1 - r0, -1)
            got = t.init_scale[r0:r1].cpu().numpy()
            assert np.array_equal(got.view(np.uint32), expect.view(np.uint32)), m.path


def test_searched_tuning_loop_matches_oracle(env):
    """A 20-step searched loop against the oracle's, from the same searched scales.

    Signed steps on beta move a whole group's scale by lr0 = 5 % at a time, so
    a gradient sign that differs between two float32 summation orders sends the
    two loops down different (equally good) paths; the final loss of one
    seed's loop therefore scatters by a few percent around the oracle's.  The
    2 % bar is applied to the mean over three calibration seeds (each loop
    within 6 %), with the initial losses matching to 1e-3.
    """
    A, SM = env
    from mround_b200.pipeline.block import DeviceBlock
    from mround_b200.pipeline.runner import QuantizationRunner, _Meter
    from mround_b200.schemes import TuningConfig

    arch = A.get_arch("tiny-qwen2")
    params = SM(arch, seed=11).block(0)
    bits, group, iters = 2, 32, 20
    scheme = scheme_for("searched", bits, group)
    finals_d, finals_o = [], []
    for seed in (2, 3, 4):
        inputs = make_inputs(arch, 4, 2, 64, seed=seed)
        dense = OracleBlock(arch, params, {p: bits for p in LINEARS}, group)
        with torch.no_grad():
            targets = [dense.forward(x) for x in inputs]
        runner = QuantizationRunner(scheme, TuningConfig(iters=iters, batch_size=2, n_samples=8,
                                                         seq_len=64))
        block = DeviceBlock(arch, params)
        tuner = runner.tuner_for(block, "model.layers.0")
        dev_inputs = [x.cuda() for x in inputs]
        tuner.search(dev_inputs)
        init = device_init_scales(tuner)
        outcome = runner._tune(tuner, dev_inputs, [t.cuda() for t in targets],
                               _Meter(torch.device("cuda")))
        oracle = OracleBlock(arch, params, {p: bits for p in LINEARS}, group, symmetric=True,
                             init_scales=init)
        ref = tune_block(oracle, inputs, targets, iters=iters,
                         lr0=runner.tuning.resolved_lr(bits), suppress=True, lo=0.5, hi=1.5)
        assert outcome["initial"] == pytest.approx(ref["initial_loss"], rel=1e-3)
        assert outcome["final"] == pytest.approx(ref["final_loss"], rel=0.06)
        assert outcome["final"] < outcome["initial"]
        finals_d.append(outcome["final"])
        finals_o.append(ref["final_loss"])
        print("searched loop seed", seed, "device", outcome["final"], "oracle", ref["final_loss"])
        layers = tuner.commit()
        assert set(layers) == set(LINEARS)
        assert all(q.scheme.scale_init.value == "searched" for q in layers.values())
    assert np.mean(finals_d) == pytest.approx(np.mean(finals_o), rel=0.02)
