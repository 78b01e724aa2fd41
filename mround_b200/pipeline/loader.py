"""Local Hugging Face checkpoints of the Llama and Qwen2 decoder families.

Replaces the reference's ``load_model`` (mround/pipeline/loader.py:176-269),
which hands the directory to mlx-lm, for the tuning path: ``config.json`` plus
``model.safetensors`` or a sharded ``model.safetensors.index.json`` in a local
directory (there is no network for Hub downloads).  Tensors are read lazily
from the files through memory maps, one block at a time, as the reference's
lazy load does, and served through the same interface as
:class:`mround_b200.pipeline.model.SyntheticModel` (``arch``, ``block(i)``,
``embed_tokens``, ``lm_head``, ``final_norm``, ``config``).

Refused loudly, as the reference refuses (loader.py:245-254) or because the
device path does not implement them: a checkpoint that is already quantized
(``quantization`` / ``quantization_config`` in its configuration), a model type
other than ``llama`` / ``qwen2``, RoPE scaling, and block linears not stored
in bf16 (the tuning kernels read bf16 weights; converting fp16 or fp32 weights
would change the model being quantized).
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np
import torch

from mround_b200.exceptions import ArchitectureError
from mround_b200.pipeline.arch import Arch
from mround_b200.pipeline.model import BlockParams

__all__ = ["CheckpointModel", "is_checkpoint_dir"]

_NP = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32}
_LINEARS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
            "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def is_checkpoint_dir(path: str | Path) -> bool:
    p = Path(path)
    return p.is_dir() and (p / "config.json").is_file()


class _SafetensorsFile:
    """Header of one safetensors file; tensors come back as memory-mapped views."""

    def __init__(self, path: Path) -> None:
        self.path = path
        with open(path, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(n))
        self.base = 8 + n
        header.pop("__metadata__", None)
        self.entries = header
        self._map: np.memmap | None = None

    def get(self, name: str) -> tuple[str, np.ndarray]:
        e = self.entries[name]
        tag = e["dtype"]
        if tag not in _NP:
            raise ArchitectureError(f"{self.path.name}: tensor {name} has dtype {tag}, "
                                    "not a floating checkpoint dtype")
        if self._map is None:
            self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        start, stop = e["data_offsets"]
        raw = self._map[self.base + start:self.base + stop]
        return tag, raw.view(_NP[tag]).reshape(e["shape"])


class CheckpointModel:
    """A Llama/Qwen2 causal LM read from a local checkpoint directory."""

    def __init__(self, path: str | Path) -> None:
        self.path = Path(path)
        cfg_file = self.path / "config.json"
        try:
            config = json.loads(cfg_file.read_text(encoding="utf-8"))
        except (OSError, ValueError) as exc:
            raise ArchitectureError(f"could not read a model configuration from {cfg_file}: {exc}") from exc
        if not isinstance(config, dict):
            raise ArchitectureError(f"{cfg_file} is not a model configuration")
        for key in ("quantization", "quantization_config"):
            if config.get(key) is not None:
                raise ArchitectureError(
                    f"{str(self.path)!r} is already quantized ({config[key]}). Quantize from the "
                    "full-precision model instead.")
        family = config.get("model_type")
        if family not in ("llama", "qwen2"):
            raise ArchitectureError(f"model_type {family!r} is not supported; the B200 path "
                                    "implements the llama and qwen2 decoder layers")
        if config.get("rope_scaling"):
            raise ArchitectureError(f"rope_scaling {config['rope_scaling']} is not implemented "
                                    "by the device block")
        if config.get("use_sliding_window"):
            raise ArchitectureError(f"use_sliding_window with sliding_window="
                                    f"{config.get('sliding_window')} is not implemented by the "
                                    "device block (its attention is fully causal)")
        # The device block applies biases to q/k/v only (Qwen2).  Llama's
        # attention_bias also gives o_proj a bias, and mlp_bias gives the three
        # MLP projections one: dropping them would tune a different function.
        if family == "llama" and config.get("attention_bias"):
            raise ArchitectureError("attention_bias=true gives the llama o_proj a bias, which the "
                                    "device block does not apply")
        if config.get("mlp_bias"):
            raise ArchitectureError("mlp_bias=true (biases on gate/up/down_proj) is not "
                                    "implemented by the device block")
        # transformers >= 5 writes the rotary settings as ``rope_parameters``
        # ({"rope_type", "rope_theta", ...}) instead of top-level keys
        rope = config.get("rope_parameters") or {}
        if rope.get("rope_type", "default") != "default":
            raise ArchitectureError(f"rope_parameters {rope} (rope_type "
                                    f"{rope.get('rope_type')!r}) is not implemented by the "
                                    "device block")
        theta = config.get("rope_theta")
        if theta is None:
            theta = rope.get("rope_theta", 10000.0)
        self._config = config
        heads = int(config["num_attention_heads"])
        hidden = int(config["hidden_size"])
        self.arch = Arch(
            name=self.path.name, family=family, hidden=hidden,
            layers=int(config["num_hidden_layers"]), heads=heads,
            kv_heads=int(config.get("num_key_value_heads", heads)),
            head_dim=int(config.get("head_dim") or hidden // heads),
            intermediate=int(config["intermediate_size"]), vocab=int(config["vocab_size"]),
            rms_eps=float(config.get("rms_norm_eps", 1e-6)),
            rope_theta=float(theta),
            qkv_bias=family == "qwen2",
            tied=bool(config.get("tie_word_embeddings", False)))
        self._files: dict[str, _SafetensorsFile] = {}
        self._where: dict[str, str] = {}
        index = self.path / "model.safetensors.index.json"
        if index.is_file():
            weight_map = json.loads(index.read_text(encoding="utf-8"))["weight_map"]
            self._where = dict(weight_map)
        elif (self.path / "model.safetensors").is_file():
            f = self._file("model.safetensors")
            self._where = {name: "model.safetensors" for name in f.entries}
        else:
            raise ArchitectureError(f"{self.path} holds no model.safetensors or index")
        if "lm_head.weight" not in self._where and not self.arch.tied:
            raise ArchitectureError("the checkpoint has no lm_head.weight and does not tie it "
                                    "to the embedding")
        self._embed: torch.Tensor | None = None

    # ------------------------------------------------------------ tensors
    def _file(self, name: str) -> _SafetensorsFile:
        if name not in self._files:
            self._files[name] = _SafetensorsFile(self.path / name)
        return self._files[name]

    def has(self, name: str) -> bool:
        return name in self._where

    def tensor(self, name: str, *, require_bf16: bool = False) -> torch.Tensor:
        """One stored tensor as bf16 (norms and biases in other float dtypes are
        rounded to bf16; linears must already be bf16 when ``require_bf16``)."""
        if name not in self._where:
            raise ArchitectureError(f"the checkpoint has no tensor {name!r}")
        tag, arr = self._file(self._where[name]).get(name)
        if tag == "BF16":
            return torch.from_numpy(np.array(arr).view(np.int16)).view(torch.bfloat16)
        if require_bf16:
            raise ArchitectureError(f"{name} is stored as {tag}; the B200 tuning path quantizes "
                                    "bf16 weights")
        return torch.from_numpy(np.array(arr)).to(torch.bfloat16)

    # ------------------------------------------------------------ model interface
    @property
    def name(self) -> str:
        return str(self.path)

    def block_name(self, index: int) -> str:
        return f"model.layers.{index}"

    def block(self, index: int) -> BlockParams:
        prefix = self.block_name(index)
        shapes = self.arch.linear_shapes()
        linears = {}
        for path in _LINEARS:
            w = self.tensor(f"{prefix}.{path}.weight", require_bf16=True)
            if tuple(w.shape) != shapes[path]:
                raise ArchitectureError(f"{prefix}.{path}.weight has shape {tuple(w.shape)}, "
                                        f"the configuration says {shapes[path]}")
            linears[path] = w
        biases = {}
        for path in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"):
            if self.has(f"{prefix}.{path}.bias"):
                biases[path] = self.tensor(f"{prefix}.{path}.bias")
        if self.arch.qkv_bias and len(biases) != 3:
            raise ArchitectureError(f"{prefix}: the architecture has q/k/v biases but the "
                                    "checkpoint does not")
        if not self.arch.qkv_bias and biases:
            raise ArchitectureError(f"{prefix}: the checkpoint carries q/k/v biases the "
                                    f"{self.arch.family} configuration does not declare")
        for path in ("self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
            if self.has(f"{prefix}.{path}.bias"):
                raise ArchitectureError(f"{prefix}.{path}.bias: the device block applies no bias "
                                        "to this projection")
        return BlockParams(index, linears, biases,
                           self.tensor(f"{prefix}.input_layernorm.weight"),
                           self.tensor(f"{prefix}.post_attention_layernorm.weight"))

    def embed_tokens(self) -> torch.Tensor:
        if self._embed is None:
            self._embed = self.tensor("model.embed_tokens.weight")
        return self._embed

    def lm_head(self) -> torch.Tensor:
        if self.arch.tied or not self.has("lm_head.weight"):
            return self.embed_tokens()
        return self.tensor("lm_head.weight")

    def final_norm(self) -> torch.Tensor:
        return self.tensor("model.norm.weight")

    def config(self) -> dict:
        return dict(self._config)
