"""Pipeline on the GPU: DeltaLoss scoring, api.quantize end to end, mixed precision.

- Scoring: per-layer per-width ``sum |g * (RTN_b(W) - W)|`` from the device's
  whole-model backward against a CPU float32 autograd oracle of the same model
  (reference mround/pipeline/scoring.py:183-311), rel 1e-3.
- api.quantize writes an MLX checkpoint whose round-to-nearest remainder
  (the embedding) is bit-exact against the oracle packer, whose block layers
  decode to in-range codes, and whose run record carries the reference's keys.
- A mixed run plans, tunes at the planned widths and records them per layer.
- BASELINE configuration 1 (SmolLM2-135M architecture, W4 asym g64, 32 x 512
  Zipf tokens, 50 iterations per block) runs end to end over all 30 blocks.
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


def _oracle_scores(model, batches, widths, group):
    from oracle.block_tuner import LINEARS, OracleBlock, rms_norm
    from oracle.deltaloss import delta_loss, rtn

    arch = model.arch
    blocks = [OracleBlock(arch, model.block(i), {p: 2 for p in LINEARS}, group)
              for i in range(arch.layers)]
    embed = model.embed_tokens().float()
    scores = {}
    for bits in widths:
        anchors = []
        for blk in blocks:
            blk.committed = {p: torch.from_numpy(rtn(blk.w[p].numpy(), bits, group)).requires_grad_(True)
                             for p in LINEARS}
            anchors.append(blk.committed)
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
            for i, blk in enumerate(blocks):
                for p in LINEARS:
                    key = f"model.layers.{i}.{p}"
                    acc[key] = acc.get(key, 0.0) + delta_loss(blk.w[p].numpy(), blk.committed[p].grad.numpy(),
                                                              bits, group)
        for key, v in acc.items():
            scores.setdefault(key, {})[bits] = v
    return scores


@pytest.mark.parametrize("seq", [33, 30])
def test_scoring_matches_oracle(seq):
    from mround_b200.pipeline.arch import get_arch
    from mround_b200.pipeline.model import SyntheticModel, zipf_tokens
    from mround_b200.pipeline.scoring import score_widths
    from mround_b200.schemes import QuantScheme

    model = SyntheticModel(get_arch("tiny-qwen2"), seed=4)
    tokens = zipf_tokens(model.arch.vocab, 2, seq, seed=1)
    batches = [tokens[0:1], tokens[1:2]]
    scheme = QuantScheme(bits=4, group_size=32, symmetry="asym")
    got = score_widths(model, batches, (2, 3, 4), scheme, gradient_source="own_width")
    want = _oracle_scores(model, batches, (2, 3, 4), 32)
    assert set(got.scores) == set(want)
    for key in want:
        for bits in (2, 3, 4):
            assert got.scores[key][bits] == pytest.approx(want[key][bits], rel=1e-3), (key, bits)
    widest = score_widths(model, batches, (2, 3, 4), scheme, gradient_source="widest")
    for key in want:  # at the widest width the two procedures coincide
        assert widest.scores[key][4] == pytest.approx(got.scores[key][4], rel=1e-6)


def test_quantize_end_to_end(tmp_path):
    from mround_b200.api import quantize
    from mround_b200.formats.safetensors_io import read_safetensors
    from mround_b200.pipeline.arch import get_arch
    from mround_b200.pipeline.model import SyntheticModel
    from mround_b200.schemes import TuningConfig
    from oracle import packing as o_pack
    from oracle import quant_fp32 as o_q

    tuning = TuningConfig(iters=10, n_samples=8, seq_len=64, batch_size=2)
    res = quantize("synthetic:tiny-qwen2", output_dir=tmp_path, bits=2, group_size=32,
                   symmetry="asym", tuning=tuning, progress=None)
    assert res.summary is not None and len(res.summary.blocks) == 2
    record = json.loads((tmp_path / "mround_run.json").read_text())
    for key in ("model", "scheme", "tuning", "calibration", "mixed", "result"):
        assert key in record
    assert record["result"]["blocks"] == 2
    arrays, tags, meta = read_safetensors(tmp_path / "model.safetensors")
    assert meta == {"format": "mlx"}
    model = SyntheticModel(get_arch("tiny-qwen2"))
    e = model.embed_tokens().float().numpy()
    ng = e.shape[1] // 32
    ones = np.ones((e.shape[0], ng), np.float32)
    _, codes, scale, zp = o_q.fake_quantize(e, np.zeros_like(e), ones, ones, 2, 32)
    assert np.array_equal(arrays["model.embed_tokens.weight"], o_pack.pack_codes(codes.astype(np.int64), 2))
    s_bits, b_bits = o_pack.to_affine(scale, zp)
    assert np.array_equal(arrays["model.embed_tokens.scales"], s_bits)
    assert np.array_equal(arrays["model.embed_tokens.biases"], b_bits)
    w = arrays["model.layers.1.mlp.down_proj.weight"]
    assert tags["model.layers.1.mlp.down_proj.weight"] == "U32"
    c = o_pack.unpack_codes(w, get_arch("tiny-qwen2").intermediate, 2)
    assert c.min() >= 0 and c.max() <= 3
    config = json.loads((tmp_path / "config.json").read_text())
    assert config["quantization"]["bits"] == 2


def test_mixed_precision_run(tmp_path):
    from mround_b200.api import quantize
    from mround_b200.schemes import TuningConfig

    tuning = TuningConfig(iters=4, n_samples=4, seq_len=64, batch_size=2)
    res = quantize("synthetic:tiny-llama", output_dir=tmp_path, bits=4, group_size=32,
                   symmetry="asym", average_bits=2.5, candidate_bits=(2, 3, 4), tuning=tuning,
                   scoring_samples=4, scoring_seq_len=64, progress=None)
    assert res.mixed is not None
    assert res.mixed["total_cost_bits"] <= res.mixed["budget_bits"]
    assigned = res.mixed["assignments"]
    assert set(assigned.values()) <= {2, 3, 4}
    for path, bits in assigned.items():
        assert res.scheme_by_layer[path].bits == bits
    config = json.loads((tmp_path / "config.json").read_text())
    q = config["quantization"]
    for path, bits in assigned.items():
        assert q.get(path, {"bits": q["bits"]})["bits"] == bits


def test_smollm2_config1_end_to_end(tmp_path):
    """BASELINE configuration 1, whole model."""
    import time

    from mround_b200.api import quantize
    from mround_b200.schemes import TuningConfig

    tuning = TuningConfig(iters=50, n_samples=32, seq_len=512, batch_size=8)
    t0 = time.perf_counter()
    res = quantize("synthetic:smollm2-135m", output_dir=tmp_path, bits=4, group_size=64,
                   symmetry="asym", tuning=tuning, progress=None)
    seconds = time.perf_counter() - t0
    print(f"smollm2-135m W4 asym g64, 30 blocks x 50 it: {seconds:.1f} s total, "
          f"loop {res.summary.total_seconds:.1f} s; {res.summary.describe()}")
    assert len(res.summary.blocks) == 30
    assert res.summary.mean_improvement > 0.0
    assert all(b.final_loss <= b.initial_loss for b in res.summary.blocks)


def test_quantize_from_checkpoint_directory_matches_synthetic(tmp_path):
    """A local HF checkpoint holding the same weights gives the same checkpoint,
    tensor for tensor, as the synthetic model (the pipeline is deterministic)."""
    from mround_b200.api import quantize
    from mround_b200.formats.safetensors_io import read_safetensors
    from mround_b200.schemes import TuningConfig
    from tests.test_loader import write_checkpoint

    ck = tmp_path / "ck"
    ck.mkdir()
    write_checkpoint(ck, "tiny-qwen2", seed=3)
    tuning = TuningConfig(iters=6, n_samples=4, seq_len=64, batch_size=2)
    out_a, out_b = tmp_path / "a", tmp_path / "b"
    quantize(str(ck), output_dir=out_a, bits=2, group_size=32, symmetry="asym", tuning=tuning,
             progress=None)
    quantize("synthetic:tiny-qwen2@3", output_dir=out_b, bits=2, group_size=32, symmetry="asym",
             tuning=tuning, progress=None)
    a, _, _ = read_safetensors(out_a / "model.safetensors")
    b, _, _ = read_safetensors(out_b / "model.safetensors")
    assert set(a) == set(b)
    for name in a:
        assert np.array_equal(a[name], b[name]), name


def test_resume_continues_a_stopped_run(tmp_path):
    """A run stopped after block 0 and restarted with the same resume
    directory writes the same checkpoint, tensor for tensor, as a run that was
    never stopped (block 0 is loaded, not re-tuned); a run with other settings
    refuses the directory."""
    from mround_b200.api import quantize
    from mround_b200.exceptions import ResumeError
    from mround_b200.formats.safetensors_io import read_safetensors
    from mround_b200.schemes import TuningConfig

    tuning = TuningConfig(iters=6, n_samples=4, seq_len=64, batch_size=2)
    kw = dict(bits=2, group_size=32, symmetry="asym", tuning=tuning)
    full, part, rdir = tmp_path / "full", tmp_path / "part", tmp_path / "resume"
    quantize("synthetic:tiny-qwen2@5", output_dir=full, progress=None, **kw)

    class Stop(Exception):
        pass

    def stop_after_block_0(line):
        if line.startswith("block   0"):
            raise Stop

    with pytest.raises(Stop):
        quantize("synthetic:tiny-qwen2@5", output_dir=part, progress=stop_after_block_0,
                 resume_dir=rdir, **kw)
    assert sorted(p.name for p in rdir.glob("block_*.pt")) == ["block_0000.pt"]
    lines = []
    quantize("synthetic:tiny-qwen2@5", output_dir=part, progress=lines.append, resume_dir=rdir,
             **kw)
    assert sorted(p.name for p in rdir.glob("block_*.pt")) == ["block_0000.pt", "block_0001.pt"]
    assert len([ln for ln in lines if ln.startswith("block")]) == 2
    a, _, _ = read_safetensors(full / "model.safetensors")
    b, _, _ = read_safetensors(part / "model.safetensors")
    assert set(a) == set(b)
    for name in a:
        assert np.array_equal(a[name], b[name]), name
    with pytest.raises(ResumeError):
        quantize("synthetic:tiny-qwen2@5", output_dir=part, progress=None, resume_dir=rdir,
                 bits=2, group_size=32, symmetry="asym",
                 tuning=TuningConfig(iters=7, n_samples=4, seq_len=64, batch_size=2))
