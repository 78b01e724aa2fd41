"""Whole-recipe parity on one Qwen2.5-0.5B block (configuration 3), opt-in.

The benchmark recipe -- W2 asym g64, 200 signSGD steps at lr 1/200, batches of
8 x 2048 tokens, outlier suppression on -- run by the CPU float32 oracle
(``oracle.block_tuner.tune_block``) and by the device runner with both
precision forms; the final block loss must agree within 2 %
(mround/pipeline/runner.py:790-953).  The oracle needs several minutes of CPU
at this size, so the test runs only when ``MR_RECIPE_TEST=1`` is set:

    MR_RECIPE_TEST=1 python -m pytest tests/test_gpu_recipe.py -m gpu -s
"""

from __future__ import annotations

import os
import time

import pytest
import torch

from oracle.block_tuner import LINEARS, OracleBlock, tune_block

pytestmark = pytest.mark.gpu

N_BATCHES, BATCH, SEQ, ITERS = 4, 8, 2048, 200


@pytest.mark.skipif(os.environ.get("MR_RECIPE_TEST") != "1",
                    reason="whole-recipe oracle loop takes minutes of CPU (set MR_RECIPE_TEST=1)")
def test_recipe_final_loss_matches_oracle():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mround_b200.pipeline.arch import get_arch
    from mround_b200.pipeline.block import TUNING_PRECISION, DeviceBlock, Precision
    from mround_b200.pipeline.model import SyntheticModel, zipf_tokens
    from mround_b200.pipeline.runner import QuantizationRunner
    from mround_b200.schemes import QuantScheme, TuningConfig

    arch = get_arch("qwen2.5-0.5b")
    model = SyntheticModel(arch, seed=0)
    embed = model.embed_tokens()
    tokens = zipf_tokens(arch.vocab, N_BATCHES * BATCH, SEQ, seed=42)
    inputs = [embed[torch.as_tensor(tokens[i * BATCH:(i + 1) * BATCH], dtype=torch.long)].float()
              for i in range(N_BATCHES)]
    params = model.block(0)
    oracle = OracleBlock(arch, params, {p: 2 for p in LINEARS}, 64)
    with torch.no_grad():
        targets = [oracle.forward(x) for x in inputs]
    t0 = time.perf_counter()
    ref = tune_block(oracle, inputs, targets, iters=ITERS, lr0=1.0 / ITERS, suppress=True)
    print(f"[recipe] oracle: {ref['initial_loss']:.6e} -> {ref['final_loss']:.6e} "
          f"({time.perf_counter() - t0:.0f} s)")
    for name, prec in (("bf16x3", Precision()), ("tuning", TUNING_PRECISION)):
        runner = QuantizationRunner(QuantScheme(bits=2, group_size=64, symmetry="asym"),
                                    TuningConfig(iters=ITERS, batch_size=BATCH,
                                                 n_samples=N_BATCHES * BATCH, seq_len=SEQ),
                                    precision=prec)
        res, _ = runner.quantize_block(DeviceBlock(arch, params), "model.layers.0",
                                       [x.cuda() for x in inputs], [t.cuda() for t in targets])
        rel = (res.final_loss - ref["final_loss"]) / ref["final_loss"]
        print(f"[recipe] device {name}: {res.initial_loss:.6e} -> {res.final_loss:.6e} "
              f"(final {rel:+.2e} of the oracle's)")
        assert abs(res.initial_loss - ref["initial_loss"]) <= 1e-3 * ref["initial_loss"]
        assert abs(rel) <= 0.02
