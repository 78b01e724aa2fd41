"""The symmetric and searched schemes through the pipeline: DeltaLoss scoring,
``api.quantize`` with the reference's default scheme, and a mixed run.

- Scoring under a searched scheme: the anchors and perturbations use each
  layer's unweighted searched scale at every width (reference
  mround/pipeline/scoring.py:195-235), against the CPU float32 autograd
  oracle, rel 1e-3.
- ``api.quantize`` with ``symmetry`` left at its default ("sym") and 2 bits
  resolves to the searched scale (reference mround/api.py:116-153): the
  round-to-nearest remainder is bit-exact against the oracle packer with the
  oracle's search, block layers carry the searched scheme and spent time in
  the search stage, stored codes are the signed codes plus 2^(b-1).
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _oracle_scores_searched(model, batches, widths, group):
    from oracle import scale_search as o_s
    from oracle.block_tuner import LINEARS, OracleBlock, rms_norm
    from oracle.deltaloss import delta_loss, rtn

    arch = model.arch
    blocks = [OracleBlock(arch, model.block(i), {p: 2 for p in LINEARS}, group)
              for i in range(arch.layers)]
    embed = model.embed_tokens().float()
    scores = {}
    for bits in widths:
        grids = [{p: o_s.search_scales_f32(blk.w[p].numpy(), bits, group).reshape(blk.w[p].shape[0], -1)
                  for p in LINEARS} for blk in blocks]
        for blk, gr in zip(blocks, grids):
            blk.committed = {p: torch.from_numpy(rtn(blk.w[p].numpy(), bits, group, symmetric=True,
                                                     init_scale=gr[p])).requires_grad_(True)
                             for p in LINEARS}
        acc = {}
        for batch in batches:
            tok = torch.as_tensor(batch, dtype=torch.long)
            x = embed[tok[:, :-1]]
            for blk in blocks:
                x = blk.forward(x)
            h = rms_norm(x, model.final_norm().float(), arch.rms_eps)
            logits = h @ embed.t()
            loss = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), tok[:, 1:].reshape(-1))
            for blk in blocks:
                for t in blk.committed.values():
                    t.grad = None
            loss.backward()
            for i, (blk, gr) in enumerate(zip(blocks, grids)):
                for p in LINEARS:
                    key = f"model.layers.{i}.{p}"
                    acc[key] = acc.get(key, 0.0) + delta_loss(
                        blk.w[p].numpy(), blk.committed[p].grad.numpy(), bits, group,
                        symmetric=True, init_scale=gr[p])
        for key, v in acc.items():
            scores.setdefault(key, {})[bits] = v
    return scores


def test_scoring_searched_matches_oracle():
    from mround_b200.pipeline.arch import get_arch
    from mround_b200.pipeline.model import SyntheticModel, zipf_tokens
    from mround_b200.pipeline.scoring import score_widths
    from mround_b200.schemes import QuantScheme

    model = SyntheticModel(get_arch("tiny-qwen2"), seed=4)
    tokens = zipf_tokens(model.arch.vocab, 2, 33, seed=1)
    batches = [tokens[0:1], tokens[1:2]]
    scheme = QuantScheme(bits=4, group_size=32, symmetry="sym", scale_init="searched")
    got = score_widths(model, batches, (2, 3, 4), scheme, gradient_source="own_width")
    want = _oracle_scores_searched(model, batches, (2, 3, 4), 32)
    assert set(got.scores) == set(want)
    for key in want:
        for bits in (2, 3, 4):
            assert got.scores[key][bits] == pytest.approx(want[key][bits], rel=1e-3), (key, bits)


def test_quantize_default_scheme_searched_end_to_end(tmp_path):
    from mround_b200.api import quantize
    from mround_b200.formats.safetensors_io import read_safetensors
    from mround_b200.pipeline.arch import get_arch
    from mround_b200.pipeline.model import SyntheticModel
    from mround_b200.schemes import TuningConfig
    from oracle import packing as o_pack
    from oracle import quant_fp32 as o_q
    from oracle import scale_search as o_s

    tuning = TuningConfig(iters=10, n_samples=8, seq_len=64, batch_size=2)
    res = quantize("synthetic:tiny-qwen2", output_dir=tmp_path, bits=2, group_size=32,
                   tuning=tuning, progress=None)
    assert res.summary is not None and len(res.summary.blocks) == 2
    assert all(b.search_seconds > 0.0 for b in res.summary.blocks)
    assert all(s.scale_init.value == "searched" and s.symmetry.value == "sym"
               for s in res.scheme_by_layer.values())
    record = json.loads((tmp_path / "mround_run.json").read_text())
    assert record["scheme"]["scale_init"] == "searched"
    arrays, tags, _ = read_safetensors(tmp_path / "model.safetensors")
    # the remainder: round-to-nearest on the unweighted searched scale
    e = SyntheticModel(get_arch("tiny-qwen2")).embed_tokens().float().numpy()
    ng = e.shape[1] // 32
    ones = np.ones((e.shape[0], ng), np.float32)
    init = o_s.search_scales_f32(e, 2, 32).reshape(e.shape[0], ng)
    _, codes, scale, _ = o_q.fake_quantize(e, np.zeros_like(e), ones, ones, 2, 32, symmetric=True,
                                           init_scale=init)
    assert np.array_equal(arrays["model.embed_tokens.weight"],
                          o_pack.pack_codes((codes + 2).astype(np.int64), 2))
    s_bits, b_bits = o_pack.to_affine(scale, None, 2)
    assert np.array_equal(arrays["model.embed_tokens.scales"], s_bits)
    assert np.array_equal(arrays["model.embed_tokens.biases"], b_bits)
    c = o_pack.unpack_codes(arrays["model.layers.1.mlp.down_proj.weight"],
                            get_arch("tiny-qwen2").intermediate, 2)
    assert c.min() >= 0 and c.max() <= 3
    assert json.loads((tmp_path / "config.json").read_text())["quantization"]["bits"] == 2


def test_quantize_symmetric_observed_4bit(tmp_path):
    from mround_b200.api import quantize
    from mround_b200.schemes import TuningConfig

    tuning = TuningConfig(iters=6, n_samples=4, seq_len=64, batch_size=2)
    res = quantize("synthetic:tiny-llama", output_dir=tmp_path, bits=4, group_size=32,
                   tuning=tuning, progress=None)
    assert all(s.scale_init.value == "observed_range" for s in res.scheme_by_layer.values())
    assert all(b.search_seconds == 0.0 for b in res.summary.blocks)


def test_mixed_precision_symmetric_run(tmp_path):
    from mround_b200.api import quantize
    from mround_b200.schemes import TuningConfig

    tuning = TuningConfig(iters=4, n_samples=4, seq_len=64, batch_size=2)
    res = quantize("synthetic:tiny-llama", output_dir=tmp_path, bits=4, group_size=32,
                   average_bits=2.5, candidate_bits=(2, 3, 4), tuning=tuning,
                   scoring_samples=4, scoring_seq_len=64, progress=None)
    assert res.mixed is not None
    assert res.mixed["total_cost_bits"] <= res.mixed["budget_bits"]
    for path, bits in res.mixed["assignments"].items():
        scheme = res.scheme_by_layer[path]
        assert scheme.bits == bits and scheme.scale_init.value == "searched"
