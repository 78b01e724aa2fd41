"""Host-side surface: schemes, recipe, CLI, refusals, the MLX checkpoint writer.

Mirrors the reference's scheme and API-default tests
(tests/unit/test_schemes.py, test_api_defaults.py) where the behaviour is the
same, and pins the checkpoint layout of mround/formats/mlx_export.py:310-425.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from mround_b200.exceptions import SchemeError, UnsupportedSchemeError
from mround_b200.schemes import QuantScheme, ScaleInit, Symmetry, TuningConfig


class TestSchemes:
    def test_defaults(self):
        s = QuantScheme()
        assert (s.bits, s.group_size, s.symmetry, s.scale_init) == (4, 64, Symmetry.SYMMETRIC,
                                                                     ScaleInit.OBSERVED_RANGE)

    @pytest.mark.parametrize("bits", [1, 9, 16])
    def test_bad_bits(self, bits):
        with pytest.raises(SchemeError):
            QuantScheme(bits=bits)

    def test_strings_are_coerced(self):
        s = QuantScheme(symmetry="asym")
        assert s.symmetry is Symmetry.ASYMMETRIC

    def test_code_ranges_and_bounds(self):
        assert QuantScheme(bits=2, symmetry="asym").code_range == (0, 3)
        assert QuantScheme(bits=4).code_range == (-8, 7)
        assert QuantScheme(bits=3, symmetry="asym").coefficient_bounds == (0.1, 1.0)
        assert QuantScheme(bits=3, scale_init="searched").coefficient_bounds == (0.5, 1.5)

    def test_searched_asym_refused(self):
        with pytest.raises(SchemeError):
            QuantScheme(symmetry="asym", scale_init="searched")

    def test_groups_per_row(self):
        assert QuantScheme(group_size=64).groups_per_row(3584) == 56
        with pytest.raises(SchemeError):
            QuantScheme(group_size=64).groups_per_row(100)

    def test_learning_rate_rule(self):
        assert TuningConfig().resolved_lr(2) == 1.0 / 200
        assert TuningConfig(iters=1000).resolved_lr(2) == 2.0 / 1000
        assert TuningConfig(iters=1000).resolved_lr(4) == 1.0 / 1000
        assert TuningConfig(lr=0.3).resolved_lr(2) == 0.3

    def test_outlier_rule(self):
        assert TuningConfig().resolved_suppress_outliers(2) is True
        assert TuningConfig().resolved_suppress_outliers(4) is False

    @pytest.mark.parametrize("kw", [{"iters": 0}, {"batch_size": 0}, {"n_samples": 4},
                                    {"minmax_lr": 0.1}, {"gradient_accumulate_steps": 2},
                                    {"micro_batches": 9}])
    def test_tuning_refusals(self, kw):
        with pytest.raises(SchemeError):
            TuningConfig(**kw)


def test_block_recipe_and_pieces():
    from mround_b200.pipeline.runner import block_recipe
    from mround_b200.pipeline.tuning import piece_bounds

    sup, rates = block_recipe(TuningConfig(), 4, {"a": 2, "b": 4}, per_layer=False)
    assert sup is False and rates == {"a": 0.005, "b": 0.005}
    sup, rates = block_recipe(TuningConfig(iters=1000), 4, {"a": 2, "b": 4}, per_layer=True)
    assert sup is True and rates == {"a": 0.002, "b": 0.001}
    assert piece_bounds(8, 3) == [(0, 3), (3, 6), (6, 8)]
    assert piece_bounds(2, 4) == [(0, 1), (1, 2)]


def test_api_resolves_every_scheme_and_refuses_bad_format():
    from mround_b200.api import _resolve_scheme, quantize
    from mround_b200.schemes import ScaleInit, Symmetry

    # the reference's defaults: symmetric, searched below 4 bits (api.py:116-153)
    s4, _ = _resolve_scheme(bits=4, group_size=64, symmetry="sym", average_bits=None,
                            candidate_bits=(), remainder_bits=None, scheme=None, scale_init=None)
    assert s4.symmetry is Symmetry.SYMMETRIC and s4.scale_init is ScaleInit.OBSERVED_RANGE
    s2, _ = _resolve_scheme(bits=2, group_size=64, symmetry="sym", average_bits=None,
                            candidate_bits=(), remainder_bits=None, scheme=None, scale_init=None)
    assert s2.scale_init is ScaleInit.SEARCHED and s2.coefficient_bounds == (0.5, 1.5)
    mixed, widths = _resolve_scheme(bits=4, group_size=64, symmetry="sym", average_bits=2.5,
                                    candidate_bits=(2, 3, 4), remainder_bits=None, scheme=None,
                                    scale_init=None)
    assert mixed.scale_init is ScaleInit.SEARCHED and widths == {2, 3, 4}
    asym, _ = _resolve_scheme(bits=2, group_size=64, symmetry="asym", average_bits=None,
                              candidate_bits=(), remainder_bits=None, scheme=None, scale_init=None)
    assert asym.scale_init is ScaleInit.OBSERVED_RANGE
    with pytest.raises(UnsupportedSchemeError):
        quantize("synthetic:tiny-qwen2", output_dir="/tmp/x", export_format="gguf")
    with pytest.raises(SchemeError):
        quantize("synthetic:tiny-qwen2", output_dir="/tmp/x", plan={"a": 2})


def test_remainder_width_ties_toward_more_bits():
    from mround_b200.api import _remainder_width

    assert _remainder_width(2.5, (2, 3, 4), None) == 3
    assert _remainder_width(3.5, (2, 3, 4), None) == 4
    assert _remainder_width(2.5, (2, 4), None) == 3
    assert _remainder_width(2.25, (2, 3, 4), 4) == 4


def test_cli_dry_run(capsys):
    from mround_b200.cli.main import main

    assert main(["quantize", "synthetic:tiny-qwen2", "-o", "/tmp/x", "--bits", "2", "--asym",
                 "--dry-run"]) == 0
    assert "asym" in capsys.readouterr().out
    # the reference's default scheme: symmetric, and searched below 4 bits
    assert main(["quantize", "synthetic:tiny-qwen2", "-o", "/tmp/x", "--dry-run"]) == 0
    assert "observed_range" in capsys.readouterr().out
    assert main(["quantize", "synthetic:tiny-qwen2", "-o", "/tmp/x", "--bits", "2",
                 "--dry-run"]) == 0
    assert "searched" in capsys.readouterr().out
    assert main(["quantize", "synthetic:tiny-qwen2", "-o", "/tmp/x", "--resume-dir", "/tmp/r",
                 "--dry-run"]) == 0


def _fake_layer(rows, cols, bits, group, seed):
    from mround_b200.pipeline.tuning import QuantizedLayer

    g = torch.Generator().manual_seed(seed)
    words = cols * bits // 32
    return QuantizedLayer(torch.randint(-2**31, 2**31 - 1, (rows, words), generator=g, dtype=torch.int32),
                          torch.randn(rows, cols // group, generator=g).to(torch.bfloat16),
                          torch.randn(rows, cols // group, generator=g).to(torch.bfloat16),
                          QuantScheme(bits=bits, group_size=group, symmetry="asym"), (rows, cols))


def test_export_layout_shards_and_index(tmp_path):
    from mround_b200.formats.mlx_export import export_mlx
    from mround_b200.formats.safetensors_io import read_safetensors

    quantized = {f"model.layers.{i}.mlp.down_proj": _fake_layer(64, 256, 2 if i else 4, 64, i)
                 for i in range(3)}
    dense = {"model.norm.weight": torch.ones(64, dtype=torch.bfloat16)}
    # stale shard from a bigger earlier export must disappear
    (tmp_path / "model-00009-of-00009.safetensors").write_bytes(b"old")
    export_mlx(tmp_path, dense, quantized, {"model_type": "qwen2"}, shard_bytes=6000)
    index = json.loads((tmp_path / "model.safetensors.index.json").read_text())
    files = sorted(set(index["weight_map"].values()))
    assert len(files) > 1 and all(f.startswith("model-") for f in files)
    assert not (tmp_path / "model-00009-of-00009.safetensors").exists()
    config = json.loads((tmp_path / "config.json").read_text())
    q = config["quantization"]
    assert q["bits"] == 2 and q["group_size"] == 64 and q["mode"] == "affine"
    assert q["model.layers.0.mlp.down_proj"] == {"group_size": 64, "bits": 4, "mode": "affine"}
    assert config["quantization_config"] == q
    seen = {}
    for f in files:
        arrays, tags, meta = read_safetensors(tmp_path / f)
        assert meta == {"format": "mlx"}
        for name, a in arrays.items():
            seen[name] = (a, tags[name])
    a, tag = seen["model.layers.1.mlp.down_proj.weight"]
    assert tag == "U32" and a.shape == (64, 16)
    assert np.array_equal(a.view(np.int32), quantized["model.layers.1.mlp.down_proj"].packed.numpy())
    assert seen["model.layers.1.mlp.down_proj.scales"][1] == "BF16"
    # a packed word counts 32/bits parameters; scales and biases count none
    want = 64 + sum(64 * 256 for _ in range(3))
    assert index["metadata"]["total_parameters"] == want


def test_export_refuses_unrepresentable(tmp_path):
    from mround_b200.formats.mlx_export import export_mlx, require_mlx_representable

    with pytest.raises(UnsupportedSchemeError):
        require_mlx_representable(QuantScheme(bits=7))
    with pytest.raises(UnsupportedSchemeError):
        require_mlx_representable(QuantScheme(group_size=-1))
    from mround_b200.exceptions import ExportError

    with pytest.raises(ExportError):
        export_mlx(tmp_path, {}, {}, {})


def test_exchange_default_follows_the_measured_rank_count():
    """The fused peer-store exchange up to four ranks, NCCL at eight (measured
    inside the 7B step); an unknown name is refused."""
    from mround_b200.pipeline.tuning import auto_exchange

    assert [auto_exchange(n) for n in (1, 2, 4, 8)] == ["p2p", "p2p", "p2p", "nccl"]


def test_k2_segments_and_codes_wrappers_refuse_before_any_launch():
    """The segmented K2 launch takes 1 to 8 matrices; CPU tensors are refused
    (no CPU fallback) before the library is called; the tuner refuses an
    unknown gather form."""
    from mround_b200 import kernels
    from mround_b200.exceptions import PlatformError

    with pytest.raises(SchemeError):
        kernels.ste_signsgd_segments([], group=64, eps=1e-8)
    with pytest.raises(SchemeError):
        kernels.ste_signsgd_segments([{}] * (kernels.MAX_K2_SEGMENTS + 1), group=64, eps=1e-8)
    w = torch.zeros(4, 64, dtype=torch.bfloat16)
    seg = {"gq": torch.zeros(4, 64), "w": w, "v": torch.zeros(4, 64), "alpha": torch.ones(4, 1),
           "beta": torch.ones(4, 1), "bits": 2, "lr": 0.01, "lo": 0.5, "hi": 1.0}
    with pytest.raises(PlatformError):
        kernels.ste_signsgd_segments([seg], group=64, eps=1e-8)
    with pytest.raises(PlatformError):
        kernels.dequant_split(torch.zeros(4, 64, dtype=torch.uint8), torch.ones(4), torch.zeros(4),
                              group=64, symmetric=False)
    from mround_b200.pipeline.tuning import BlockTuner

    with pytest.raises(ValueError, match="gather"):
        BlockTuner(None, {}, {}, suppress=False, eps=1e-8, precision=None, dist=None,
                   gather="rows")
