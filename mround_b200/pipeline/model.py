"""Synthetic models of the benchmark architectures, and their calibration tokens.

The benchmark configurations use random-initialised weights of the named
architectures (no checkpoints are available offline): every linear,
embedding and bias ~ N(0, 0.02), RMSNorm weights = 1, bf16 storage.  Each
tensor is drawn from its own CPU ``torch.Generator`` seeded by the model seed
and the tensor's name, so a block's weights do not depend on which other
blocks were built, and the CPU oracle and the GPU path see identical values.

Calibration tokens stand in for pile-10k (reference
``mround/pipeline/calibration.py:408-506``): a truncated Zipf law
``p(k) ~ k**-1.1`` over the vocabulary, token id = rank - 1, drawn with
``numpy.random.default_rng(seed).choice``, batched ``(batch, seq_len)``.
"""

from __future__ import annotations

import dataclasses
import hashlib

import numpy as np
import torch

from mround_b200.pipeline.arch import Arch

__all__ = ["BlockParams", "SyntheticModel", "zipf_tokens", "tensor_seed"]


def tensor_seed(seed: int, name: str) -> int:
    digest = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(digest[:8], "little") & ((1 << 63) - 1)


def _normal_bf16(shape: tuple[int, ...], seed: int, name: str, std: float = 0.02) -> torch.Tensor:
    g = torch.Generator().manual_seed(tensor_seed(seed, name))
    return (torch.randn(shape, generator=g) * std).to(torch.bfloat16)


@dataclasses.dataclass
class BlockParams:
    """Dense weights of one decoder block, keyed by mlx-lm module path.

    ``linears[path]`` is the bf16 (out, in) weight; ``biases[path]`` the bf16
    bias where the architecture has one; norms are the two RMSNorm weights.
    """

    index: int
    linears: dict[str, torch.Tensor]
    biases: dict[str, torch.Tensor]
    input_norm: torch.Tensor
    post_norm: torch.Tensor

    def to(self, device: torch.device | str) -> BlockParams:
        return BlockParams(
            self.index,
            {k: v.to(device) for k, v in self.linears.items()},
            {k: v.to(device) for k, v in self.biases.items()},
            self.input_norm.to(device),
            self.post_norm.to(device),
        )


class SyntheticModel:
    """A randomly initialised decoder of a given architecture, built lazily per block."""

    def __init__(self, arch: Arch, seed: int = 0) -> None:
        self.arch = arch
        self.seed = seed
        self._embed: torch.Tensor | None = None

    @property
    def name(self) -> str:
        return f"synthetic-{self.arch.name}"

    def block_name(self, index: int) -> str:
        return f"model.layers.{index}"

    def block(self, index: int) -> BlockParams:
        a = self.arch
        prefix = self.block_name(index)
        linears = {
            path: _normal_bf16(shape, self.seed, f"{prefix}.{path}.weight")
            for path, shape in a.linear_shapes().items()
        }
        biases = {}
        if a.qkv_bias:
            for path in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"):
                biases[path] = _normal_bf16((linears[path].shape[0],), self.seed, f"{prefix}.{path}.bias")
        ones = torch.ones(a.hidden, dtype=torch.bfloat16)
        return BlockParams(index, linears, biases, ones.clone(), ones.clone())

    def embed_tokens(self) -> torch.Tensor:
        if self._embed is None:
            self._embed = _normal_bf16((self.arch.vocab, self.arch.hidden), self.seed,
                                       "model.embed_tokens.weight")
        return self._embed

    def lm_head(self) -> torch.Tensor:
        if self.arch.tied:
            return self.embed_tokens()
        return _normal_bf16((self.arch.vocab, self.arch.hidden), self.seed, "lm_head.weight")

    def final_norm(self) -> torch.Tensor:
        return torch.ones(self.arch.hidden, dtype=torch.bfloat16)

    def config(self) -> dict:
        a = self.arch
        return {
            "model_type": a.family,
            "hidden_size": a.hidden,
            "num_hidden_layers": a.layers,
            "num_attention_heads": a.heads,
            "num_key_value_heads": a.kv_heads,
            "head_dim": a.head_dim,
            "intermediate_size": a.intermediate,
            "vocab_size": a.vocab,
            "rms_norm_eps": a.rms_eps,
            "rope_theta": a.rope_theta,
            "tie_word_embeddings": a.tied,
            "torch_dtype": "bfloat16",
        }


def zipf_tokens(vocab: int, n_samples: int, seq_len: int, seed: int = 42, s: float = 1.1) -> np.ndarray:
    """(n_samples, seq_len) int32 token ids, truncated Zipf over the vocabulary."""
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** (-s)
    p /= p.sum()
    rng = np.random.default_rng(seed)
    return rng.choice(vocab, size=(n_samples, seq_len), p=p).astype(np.int32)
