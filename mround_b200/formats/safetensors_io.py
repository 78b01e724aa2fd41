"""Minimal safetensors writer/reader (the MLX checkpoint's container).

A safetensors file is an 8-byte little-endian header length, a JSON header
mapping tensor names to ``{"dtype", "shape", "data_offsets"}`` (plus an
optional ``__metadata__`` string map), then the raw little-endian tensor bytes
back to back.  Writing it here, rather than through a framework, fixes the
dtype tags MLX expects (``U32`` for packed codes, ``BF16`` for scales and
biases) and the ``{"format": "mlx"}`` metadata mlx-lm's loader checks
(reference mround/formats/mlx_export.py:392).
"""

from __future__ import annotations

import json
import struct
from collections.abc import Mapping
from pathlib import Path

import numpy as np
import torch

__all__ = ["read_safetensors", "tensor_bytes", "write_safetensors"]

_TAGS = {
    torch.bfloat16: ("BF16", 2),
    torch.float16: ("F16", 2),
    torch.float32: ("F32", 4),
    torch.int32: ("I32", 4),
    torch.uint8: ("U8", 1),
    torch.int8: ("I8", 1),
    torch.int64: ("I64", 8),
}


def _as_bytes(t: torch.Tensor, tag_override: str | None) -> tuple[str, bytes]:
    t = t.detach().contiguous().cpu()
    tag, _ = _TAGS[t.dtype]
    if tag_override:
        tag = tag_override
    if t.dtype == torch.bfloat16:
        raw = t.view(torch.int16).numpy().tobytes()
    else:
        raw = t.numpy().tobytes()
    return tag, raw


def tensor_bytes(t: torch.Tensor) -> int:
    return t.numel() * _TAGS[t.dtype][1]


def write_safetensors(path: Path, tensors: Mapping[str, torch.Tensor], *,
                      metadata: Mapping[str, str] | None = None,
                      dtype_tags: Mapping[str, str] | None = None) -> None:
    """Write ``tensors`` in the given order.  ``dtype_tags`` overrides a tag
    (packed words are held as int32 and stored as ``U32``)."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = dict(metadata)
    blobs = []
    offset = 0
    for name, t in tensors.items():
        tag, raw = _as_bytes(t, (dtype_tags or {}).get(name))
        header[name] = {"dtype": tag, "shape": list(t.shape), "data_offsets": [offset, offset + len(raw)]}
        offset += len(raw)
        blobs.append(raw)
    text = json.dumps(header, separators=(",", ":")).encode()
    text += b" " * ((8 - len(text) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for raw in blobs:
            f.write(raw)


_NP = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32, "I32": np.int32, "U32": np.uint32,
       "U8": np.uint8, "I8": np.int8, "I64": np.int64}


def read_safetensors(path: Path) -> tuple[dict[str, np.ndarray], dict[str, str], dict[str, str]]:
    """``(arrays, dtype tags, metadata)``; bf16 arrays come back as uint16 patterns."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        base = 8 + n
        data = f.read()
    meta = header.pop("__metadata__", {})
    arrays, tags = {}, {}
    for name, info in header.items():
        a, b = info["data_offsets"]
        arrays[name] = np.frombuffer(data[a:b], dtype=_NP[info["dtype"]]).reshape(info["shape"])
        tags[name] = info["dtype"]
    del base
    return arrays, tags, meta
