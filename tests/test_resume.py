"""Per-block resume store (host side, no GPU): manifest fingerprints, block
records round-tripping through disk, refusals of foreign or damaged records."""

from __future__ import annotations

import json

import pytest
import torch

from mround_b200.exceptions import ResumeError
from mround_b200.pipeline.arch import get_arch
from mround_b200.pipeline.resume import ResumeStore, run_fingerprint, tokens_digest
from mround_b200.pipeline.runner import BlockResult
from mround_b200.pipeline.tuning import QuantizedLayer
from mround_b200.schemes import QuantScheme, TuningConfig


def _fingerprint(iters=20, tokens=None, world=1):
    tokens = tokens if tokens is not None else [[1, 2, 3, 4], [5, 6, 7, 8]]
    return run_fingerprint(model="synthetic:tiny-qwen2", arch=get_arch("tiny-qwen2"),
                           scheme=QuantScheme(bits=2, group_size=32, symmetry="asym"),
                           tuning=TuningConfig(iters=iters, n_samples=4, seq_len=64, batch_size=2),
                           scheme_by_layer=None, batches=tokens, world=world,
                           quantized_inputs=True)


def _block(index=0):
    g = torch.Generator().manual_seed(index)
    scheme = QuantScheme(bits=2, group_size=32, symmetry="asym")
    layers = {
        f"model.layers.{index}.self_attn.q_proj": QuantizedLayer(
            torch.randint(-2**31, 2**31 - 1, (128, 8), dtype=torch.int32, generator=g),
            torch.randn(128, 4, generator=g).to(torch.bfloat16),
            torch.randn(128, 4, generator=g).to(torch.bfloat16), scheme, (128, 128),
            torch.randint(0, 4, (128, 128), dtype=torch.uint8, generator=g)),
        f"model.layers.{index}.mlp.down_proj": QuantizedLayer(
            torch.randint(-2**31, 2**31 - 1, (128, 24), dtype=torch.int32, generator=g),
            torch.randn(128, 12, generator=g).to(torch.bfloat16),
            torch.randn(128, 12, generator=g).to(torch.bfloat16),
            QuantScheme(bits=3, group_size=32, symmetry="sym", scale_init="searched"),
            (128, 384)),
    }
    result = BlockResult(index=index, name=f"model.layers.{index}", initial_loss=1.5e-3,
                         final_loss=1.1e-3, iterations=20, seconds=2.5, peak_memory_bytes=123456,
                         tuned=("mlp.down_proj", "self_attn.q_proj"),
                         skipped=(("mlp.gate_proj", "why"),), reverted=False,
                         generalization_gap=None, search_seconds=0.1,
                         stage_peaks={"tune": 99}, step_seconds=0.01)
    committed = {"qkv": torch.randn(256, 128, generator=g).to(torch.bfloat16),
                 "down": torch.randn(128, 384, generator=g).to(torch.bfloat16)}
    return result, layers, committed


def test_fingerprint_tracks_calibration_and_settings():
    assert _fingerprint() == _fingerprint()
    assert _fingerprint(iters=21) != _fingerprint()
    assert _fingerprint(world=2) != _fingerprint()
    assert tokens_digest([[1, 2], [3, 4]]) != tokens_digest([[1, 2, 3, 4]])
    assert _fingerprint(tokens=[[1, 2, 3, 4], [5, 6, 7, 9]]) != _fingerprint()


def test_manifest_is_written_once_and_foreign_runs_are_refused(tmp_path):
    d = tmp_path / "resume"
    ResumeStore(d, _fingerprint())
    stored = json.loads((d / "manifest.json").read_text())
    assert stored["calibration_sha256"] == tokens_digest([[1, 2, 3, 4], [5, 6, 7, 8]])
    ResumeStore(d, _fingerprint())  # the same run continues
    with pytest.raises(ResumeError, match="tuning"):
        ResumeStore(d, _fingerprint(iters=50))
    with pytest.raises(ResumeError, match="calibration_sha256"):
        ResumeStore(d, _fingerprint(tokens=[[9, 9, 9, 9], [5, 6, 7, 8]]))


def test_block_records_round_trip(tmp_path):
    store = ResumeStore(tmp_path / "r", _fingerprint())
    for index in (0, 1):
        result, layers, committed = _block(index)
        store.save(index, result, layers, committed)
    assert store.completed() == [0, 1]
    assert not list((tmp_path / "r").glob("*.tmp*"))
    again = ResumeStore(tmp_path / "r", _fingerprint())
    result, layers, committed = _block(1)
    stored = again.load(1)
    assert stored.result["final_loss"] == result.final_loss
    assert stored.result["tuned"] == list(result.tuned)
    for name, t in committed.items():
        assert stored.committed[name].dtype == torch.bfloat16
        assert torch.equal(stored.committed[name], t)
    rebuilt = ResumeStore.quantized_layers(stored, QuantizedLayer)
    assert set(rebuilt) == set(layers)
    for path, q in layers.items():
        r = rebuilt[path]
        assert torch.equal(r.packed, q.packed) and torch.equal(r.scales, q.scales)
        assert torch.equal(r.biases, q.biases)
        assert r.scheme == q.scheme and r.shape == q.shape
        assert (r.codes is None) == (q.codes is None)
        if q.codes is not None:
            assert torch.equal(r.codes, q.codes)


def test_other_ranks_do_not_write(tmp_path):
    ResumeStore(tmp_path / "r", _fingerprint(), rank=0)
    store = ResumeStore(tmp_path / "r", _fingerprint(), rank=1)
    store.save(0, *_block(0))
    assert store.completed() == []


def test_damaged_and_missing_records_are_refused(tmp_path):
    store = ResumeStore(tmp_path / "r", _fingerprint())
    with pytest.raises(ResumeError, match="missing"):
        store.load(3)
    store.path(0).write_bytes(b"not a torch file")
    with pytest.raises(ResumeError, match="cannot be read"):
        store.load(0)
    torch.save({"something": 1}, store.path(1))
    with pytest.raises(ResumeError, match="not a block record"):
        store.load(1)
