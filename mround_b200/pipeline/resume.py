"""Per-block resume of a tuning run.

A long run (28 blocks of a 7B model) can be stopped and restarted without
re-tuning the blocks it finished.  After each block the runner hands this
store the block's outcome, which it writes as ``block_<index>.pt``:

* the committed layers in their stored form (packed words, bf16 scales and
  biases, the scheme, the shape, the codes when kept) -- what the export needs;
* each fused weight's committed bf16 reconstruction -- the operand the
  quantized activation stream advances through, so a restarted run rebuilds
  that stream exactly;
* the block's :class:`~mround_b200.pipeline.runner.BlockResult`.

A restarted run that finds ``block_<index>.pt`` for the next block in order
loads it, replays the block's forward passes (targets through the original
weights, the quantized stream through the committed ones) and moves on; the
first block without a file is tuned as usual.  Forward passes are a few per
cent of a block's tuning time.

``manifest.json`` records what the run is (model, architecture, schemes,
tuning configuration, a digest of the calibration tokens, rank count, ...).
A directory written by a different run is refused with
:class:`~mround_b200.exceptions.ResumeError` rather than silently mixed in.
Files are written to a temporary name and renamed, so a run stopped while
writing leaves no partial block behind.  Only rank 0 writes; every rank
reads.  Everything is stored as plain tensors, numbers and strings, loaded
with ``torch.load(weights_only=True)``.

The reference has no counterpart (its runs restart from block 0); the stored
layers are the reference's committed form (mround/pipeline/runner.py:761-788).
"""

from __future__ import annotations

import dataclasses
import hashlib
import json
import os
from collections.abc import Mapping, Sequence
from pathlib import Path
from typing import Any

import numpy as np
import torch

from mround_b200.exceptions import ResumeError
from mround_b200.schemes import QuantScheme

__all__ = ["ResumeStore", "StoredBlock", "run_fingerprint", "tokens_digest"]

MANIFEST = "manifest.json"
FORMAT = 1


def tokens_digest(batches: Sequence[Any]) -> str:
    """SHA-256 over the calibration token ids, batch by batch."""
    h = hashlib.sha256()
    for batch in batches:
        arr = np.ascontiguousarray(np.asarray(batch, dtype=np.int64))
        h.update(str(arr.shape).encode())
        h.update(arr.tobytes())
    return h.hexdigest()


def _scheme_dict(scheme: QuantScheme) -> dict[str, Any]:
    return {"bits": int(scheme.bits), "group_size": int(scheme.group_size),
            "symmetry": scheme.symmetry.value, "scale_init": scheme.scale_init.value}


def run_fingerprint(*, model: str, arch: Any, scheme: QuantScheme, tuning: Any,
                    scheme_by_layer: Mapping[str, QuantScheme] | None, batches: Sequence[Any],
                    world: int, **extra: Any) -> dict[str, Any]:
    """What two runs must share for one to continue the other's blocks."""
    overrides = None
    if scheme_by_layer is not None:
        overrides = {path: _scheme_dict(s) for path, s in sorted(scheme_by_layer.items())}
    return {
        "format": FORMAT,
        "model": str(model),
        "arch": dataclasses.asdict(arch) if dataclasses.is_dataclass(arch) else str(arch),
        "scheme": _scheme_dict(scheme),
        "scheme_by_layer": overrides,
        "tuning": dataclasses.asdict(tuning) if dataclasses.is_dataclass(tuning) else str(tuning),
        "calibration_sha256": tokens_digest(batches),
        "world": int(world),
        **{k: v for k, v in sorted(extra.items())},
    }


def _canonical(value: Any) -> Any:
    """JSON round trip, so a fingerprint compares equal to its stored copy."""
    return json.loads(json.dumps(value, sort_keys=True, default=str))


@dataclasses.dataclass
class StoredBlock:
    result: dict[str, Any]                   # BlockResult fields
    layers: dict[str, dict[str, Any]]        # path -> QuantizedLayer fields (scheme as a dict)
    committed: dict[str, torch.Tensor]       # fused weight name -> bf16 reconstruction (CPU)


class ResumeStore:
    def __init__(self, directory: str | Path, fingerprint: Mapping[str, Any], *,
                 rank: int = 0) -> None:
        self.directory = Path(directory)
        self.rank = rank
        self.fingerprint = _canonical(dict(fingerprint))
        manifest = self.directory / MANIFEST
        if manifest.exists():
            stored = json.loads(manifest.read_text(encoding="utf-8"))
            if stored != self.fingerprint:
                differing = sorted(k for k in set(stored) | set(self.fingerprint)
                                   if stored.get(k) != self.fingerprint.get(k))
                raise ResumeError(f"{self.directory} holds blocks of a different run "
                                  f"(differs in: {', '.join(differing)}); use another "
                                  f"directory or remove it")
        elif rank == 0:
            self.directory.mkdir(parents=True, exist_ok=True)
            self._write_atomic(manifest, json.dumps(self.fingerprint, indent=2, sort_keys=True)
                               .encode("utf-8"))

    # ------------------------------------------------------------ paths
    def path(self, index: int) -> Path:
        return self.directory / f"block_{index:04d}.pt"

    def has(self, index: int) -> bool:
        return self.path(index).exists()

    def completed(self) -> list[int]:
        return sorted(int(p.stem.split("_")[1]) for p in self.directory.glob("block_*.pt"))

    @staticmethod
    def _write_atomic(path: Path, payload: bytes | dict) -> None:
        """Write to a temporary name, flush to disk, then rename over ``path``
        (bytes are written as they are; a dict is written by torch.save
        straight to the file, without a second copy in host memory)."""
        tmp = path.with_name(path.name + f".tmp{os.getpid()}")
        with open(tmp, "wb") as f:
            if isinstance(payload, bytes):
                f.write(payload)
            else:
                torch.save(payload, f)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)

    # ------------------------------------------------------------ write / read
    def save(self, index: int, result: Any, layers: Mapping[str, Any],
             committed: Mapping[str, torch.Tensor]) -> None:
        """Write one finished block (rank 0 only; other ranks return)."""
        if self.rank != 0:
            return
        fields = dataclasses.asdict(result) if dataclasses.is_dataclass(result) else dict(result)
        record = {
            "result": _canonical(fields),
            "layers": {
                path: {"packed": q.packed.cpu(), "scales": q.scales.cpu(), "biases": q.biases.cpu(),
                       "scheme": _scheme_dict(q.scheme), "shape": [int(s) for s in q.shape],
                       "codes": None if q.codes is None else q.codes.cpu()}
                for path, q in layers.items()
            },
            "committed": {name: t.detach().to("cpu", copy=True).contiguous()
                          for name, t in committed.items()},
        }
        self._write_atomic(self.path(index), record)

    def load(self, index: int) -> StoredBlock:
        path = self.path(index)
        if not path.exists():
            raise ResumeError(f"{path} is missing")
        try:
            record = torch.load(path, map_location="cpu", weights_only=True)
        except Exception as exc:  # noqa: BLE001 - any unreadable file is the same refusal
            raise ResumeError(f"{path} cannot be read ({exc}); remove it to re-tune the block") from exc
        try:
            return StoredBlock(result=record["result"], layers=record["layers"],
                               committed=record["committed"])
        except (KeyError, TypeError) as exc:
            raise ResumeError(f"{path} is not a block record ({exc})") from exc

    @staticmethod
    def quantized_layers(stored: StoredBlock, layer_type: Any) -> dict[str, Any]:
        """Rebuild ``QuantizedLayer`` objects from a stored block."""
        out = {}
        for path, f in stored.layers.items():
            out[path] = layer_type(f["packed"], f["scales"], f["biases"], QuantScheme(**f["scheme"]),
                                   tuple(f["shape"]), f["codes"])
        return out
