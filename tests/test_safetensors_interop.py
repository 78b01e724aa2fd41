"""The checkpoint container against the safetensors library itself.

Our writer fixes the dtype tags MLX expects (``U32`` packed words held as
int32, ``BF16`` scales and biases) and the ``{"format": "mlx"}`` metadata;
files it writes must load with the ``safetensors`` package (the format's
reference implementation, which mlx-lm's loader also reads) with the same
values, tags and metadata, and files the package writes must read back here.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mround_b200.formats.safetensors_io import read_safetensors, write_safetensors

safetensors = pytest.importorskip("safetensors")


def _tensors():
    g = torch.Generator().manual_seed(0)
    return {
        "model.layers.0.mlp.down_proj.weight": torch.randint(-2**31, 2**31 - 1, (8, 4),
                                                             dtype=torch.int32, generator=g),
        "model.layers.0.mlp.down_proj.scales": torch.randn(8, 2, generator=g).to(torch.bfloat16),
        "model.layers.0.mlp.down_proj.biases": torch.randn(8, 2, generator=g).to(torch.bfloat16),
        "model.norm.weight": torch.randn(16, generator=g),
        "codes": torch.randint(0, 255, (3, 5), dtype=torch.uint8, generator=g),
    }


def test_our_files_load_in_safetensors(tmp_path):
    from safetensors import safe_open

    tensors = _tensors()
    packed = "model.layers.0.mlp.down_proj.weight"
    path = tmp_path / "model.safetensors"
    write_safetensors(path, tensors, metadata={"format": "mlx"}, dtype_tags={packed: "U32"})
    with safe_open(str(path), framework="np") as f:
        assert f.metadata() == {"format": "mlx"}
        assert set(f.keys()) == set(tensors)
        words = f.get_tensor(packed)
        assert words.dtype == np.uint32
        assert np.array_equal(words.view(np.int32), tensors[packed].numpy())
        for name in ("model.norm.weight", "codes"):
            assert np.array_equal(f.get_tensor(name), tensors[name].numpy())
    with safe_open(str(path), framework="pt") as f:
        for name in ("model.layers.0.mlp.down_proj.scales", "model.layers.0.mlp.down_proj.biases"):
            got = f.get_tensor(name)
            assert got.dtype == torch.bfloat16 and torch.equal(got, tensors[name])


def test_library_files_read_back_here(tmp_path):
    from safetensors.torch import save_file

    tensors = {k: v for k, v in _tensors().items()}
    path = tmp_path / "lib.safetensors"
    save_file(tensors, str(path), metadata={"format": "pt"})
    arrays, tags, meta = read_safetensors(path)
    assert meta == {"format": "pt"}
    for name, t in tensors.items():
        if t.dtype == torch.bfloat16:
            assert tags[name] == "BF16"
            assert np.array_equal(arrays[name], t.view(torch.int16).numpy().view(np.uint16))
        else:
            assert np.array_equal(arrays[name], t.numpy())
