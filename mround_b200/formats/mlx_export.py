"""MLX-format checkpoint writer for layers committed on the device.

Restates the checkpoint layout of reference mround/formats/mlx_export.py
(310-425): quantized layers as ``<path>.weight`` (packed uint32 codes),
``<path>.scales`` and ``<path>.biases`` (model dtype, ``(out, n_groups)``);
dense tensors verbatim; weight files of at most 5 GiB
(``model.safetensors`` or ``model-0000i-of-0000N.safetensors``) with
``{"format": "mlx"}`` metadata; ``model.safetensors.index.json`` with
``total_size`` and ``total_parameters`` (a packed word counts ``32 / bits``
parameters, scales and biases none); ``config.json`` extended by the
``quantization`` block (most common scheme as default, per-layer overrides)
duplicated under ``quantization_config``.  Stale weight files of an earlier
export in the same directory are removed.

The packed words, scales and biases arrive already in their stored form from
K5 (``mr_pack_mlx``), so exporting is layout and file writing only.
"""

from __future__ import annotations

import json
import re
from collections.abc import Mapping
from pathlib import Path
from typing import Any

import torch

from mround_b200.exceptions import ExportError, UnsupportedSchemeError
from mround_b200.formats.safetensors_io import tensor_bytes, write_safetensors
from mround_b200.pipeline.tuning import QuantizedLayer
from mround_b200.schemes import QuantScheme

__all__ = [
    "MLX_GROUP_SIZES",
    "MLX_SUPPORTED_BITS",
    "SHARD_BYTES",
    "export_mlx",
    "require_mlx_representable",
    "shard_names",
]

MLX_SUPPORTED_BITS = frozenset({2, 3, 4, 5, 6, 8})
MLX_GROUP_SIZES = frozenset({32, 64, 128})
RESERVED_CONFIG_KEYS = frozenset({"group_size", "bits", "mode"})
SHARD_BYTES = 5 << 30
_WEIGHT_FILE = re.compile(r"model(-\d{5}-of-\d{5})?\.safetensors")


def require_mlx_representable(scheme: QuantScheme, *, path: str = "scheme") -> None:
    if scheme.bits not in MLX_SUPPORTED_BITS:
        allowed = ", ".join(str(b) for b in sorted(MLX_SUPPORTED_BITS))
        raise UnsupportedSchemeError(
            f"{path}: MLX quantization accepts bits in {{{allowed}}} and rejects {scheme.bits}")
    if scheme.group_size not in MLX_GROUP_SIZES:
        sizes = ", ".join(str(g) for g in sorted(MLX_GROUP_SIZES))
        detail = "per-channel" if scheme.is_per_channel else str(scheme.group_size)
        raise UnsupportedSchemeError(
            f"{path}: MLX quantization accepts group sizes {{{sizes}}} and cannot represent {detail}.")


def shard_names(count: int) -> list[str]:
    if count < 1:
        raise ExportError(f"a checkpoint has at least one weight file, not {count}")
    if count == 1:
        return ["model.safetensors"]
    return [f"model-{i:05d}-of-{count:05d}.safetensors" for i in range(1, count + 1)]


def _layer_tensors(path: str, layer: QuantizedLayer, dtype: torch.dtype) -> dict[str, torch.Tensor]:
    scheme = layer.scheme
    require_mlx_representable(scheme, path=path)
    out_f, in_f = layer.shape
    words = in_f * scheme.bits // 32
    if tuple(layer.packed.shape) != (out_f, words):
        raise ExportError(f"{path}: packed to {tuple(layer.packed.shape)}, expected {(out_f, words)}")
    ng = in_f // scheme.group_size
    if tuple(layer.scales.shape) != (out_f, ng):
        raise ExportError(f"{path}: scales shaped {tuple(layer.scales.shape)}, expected {(out_f, ng)}")
    scales, biases = layer.scales, layer.biases
    if dtype != torch.bfloat16:
        # K5 rounds to bf16; another model dtype would re-derive the bias from
        # the stored scale in that dtype, which the device path does not do.
        raise ExportError("the device exporter writes bf16 scales and biases only")
    return {f"{path}.weight": layer.packed, f"{path}.scales": scales, f"{path}.biases": biases}


def _shards(tensors: Mapping[str, torch.Tensor], limit: int) -> list[dict[str, torch.Tensor]]:
    shards: list[dict[str, torch.Tensor]] = [{}]
    held = 0
    for name, t in tensors.items():
        size = tensor_bytes(t)
        if shards[-1] and held + size > limit:
            shards.append({})
            held = 0
        shards[-1][name] = t
        held += size
    return shards


def _quantization_block(quantized: Mapping[str, QuantizedLayer]) -> dict[str, Any]:
    schemes = [layer.scheme for layer in quantized.values()]
    ordered = sorted(set(schemes), key=lambda s: (s.bits, s.group_size, s.symmetry.value,
                                                 s.scale_init.value))
    default = max(ordered, key=schemes.count)
    block: dict[str, Any] = {"group_size": default.group_size, "bits": default.bits, "mode": "affine"}
    for path, layer in sorted(quantized.items()):
        if layer.scheme == default:
            continue
        if path in RESERVED_CONFIG_KEYS:
            raise ExportError(f"module path {path!r} collides with a quantization setting key")
        block[path] = {"group_size": layer.scheme.group_size, "bits": layer.scheme.bits,
                       "mode": "affine"}
    return block


def export_mlx(output_dir: Path, dense_weights: Mapping[str, torch.Tensor],
               quantized: Mapping[str, QuantizedLayer], config: Mapping[str, Any], *,
               dtype: str = "bfloat16", extra_files: Mapping[str, str] | None = None,
               shard_bytes: int = SHARD_BYTES) -> None:
    """Write an mlx-lm-loadable checkpoint."""
    dtypes = {"bfloat16": torch.bfloat16}
    if dtype not in dtypes:
        raise ExportError(f"dtype must be one of {{bfloat16}}, got {dtype!r}")
    if not quantized:
        raise ExportError("nothing to export: no quantized layers were supplied")
    target = dtypes[dtype]
    tensors: dict[str, torch.Tensor] = dict(dense_weights)
    packed_names = set()
    for path, layer in sorted(quantized.items()):
        if f"{path}.weight" in dense_weights:
            raise ExportError(f"{path}.weight appears as both a dense and a quantized tensor")
        tensors.update(_layer_tensors(path, layer, target))
        packed_names.add(f"{path}.weight")
    merged = dict(config)
    block = _quantization_block(quantized)
    merged["quantization"] = block
    merged["quantization_config"] = block
    shards = _shards(tensors, shard_bytes)
    names = shard_names(len(shards))
    weight_map = {t: f for shard, f in zip(shards, names, strict=True) for t in shard}
    try:
        output_dir.mkdir(parents=True, exist_ok=True)
        for shard, fname in zip(shards, names, strict=True):
            tags = {n: "U32" for n in shard if n in packed_names}
            write_safetensors(output_dir / fname, shard, metadata={"format": "mlx"}, dtype_tags=tags)
        for stale in output_dir.iterdir():
            if _WEIGHT_FILE.fullmatch(stale.name) and stale.name not in names:
                stale.unlink()
        (output_dir / "config.json").write_text(json.dumps(merged, indent=2) + "\n")
        meta_names = {f"{p}.{k}" for p in quantized for k in ("scales", "biases")}
        total_parameters = sum(
            t.numel() * 32 // quantized[n.removesuffix(".weight")].scheme.bits
            if n in packed_names else t.numel()
            for n, t in tensors.items() if n not in meta_names)
        index = {
            "metadata": {"total_size": sum(tensor_bytes(t) for t in tensors.values()),
                         "total_parameters": total_parameters},
            "weight_map": {n: weight_map[n] for n in sorted(weight_map)},
        }
        (output_dir / "model.safetensors.index.json").write_text(json.dumps(index, indent=2) + "\n")
        for name, content in (extra_files or {}).items():
            (output_dir / name).write_text(content)
    except OSError as exc:
        raise ExportError(f"could not write the checkpoint to {output_dir}: {exc}") from exc
