"""Decoder architectures of the benchmark configurations.

Llama (SmolLM2) and Qwen2 decoder layers as mlx-lm builds them: RMSNorm,
q/k/v projections (Qwen2 with bias), rotary embedding over the full head
dimension in the non-interleaved ("rotate half") form, causal grouped-query
attention with scale ``head_dim ** -0.5``, output projection, residual,
RMSNorm, SwiGLU MLP, residual.  The reference runs the mlx-lm layer inside
``block_output`` (mround/pipeline/blocks.py:578-606); its math is restated in
:mod:`mround_b200.pipeline.block`.
"""

from __future__ import annotations

import dataclasses

__all__ = ["ARCHITECTURES", "Arch", "get_arch"]


@dataclasses.dataclass(frozen=True, slots=True)
class Arch:
    name: str
    family: str  # "llama" or "qwen2"
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rms_eps: float
    rope_theta: float
    qkv_bias: bool
    tied: bool

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def linear_shapes(self) -> dict[str, tuple[int, int]]:
        """(out_features, in_features) of each block linear, by mlx-lm module path."""
        h, i = self.hidden, self.intermediate
        return {
            "self_attn.q_proj": (self.q_dim, h),
            "self_attn.k_proj": (self.kv_dim, h),
            "self_attn.v_proj": (self.kv_dim, h),
            "self_attn.o_proj": (h, self.q_dim),
            "mlp.gate_proj": (i, h),
            "mlp.up_proj": (i, h),
            "mlp.down_proj": (h, i),
        }

    def block_weights(self) -> int:
        """Weights in the linears of one block."""
        return sum(o * i for o, i in self.linear_shapes().values())


ARCHITECTURES: dict[str, Arch] = {
    "smollm2-135m": Arch("smollm2-135m", "llama", 576, 30, 9, 3, 64, 1536, 49152, 1e-5, 1e5,
                         False, True),
    "qwen2.5-0.5b": Arch("qwen2.5-0.5b", "qwen2", 896, 24, 14, 2, 64, 4864, 151936, 1e-6, 1e6,
                         True, True),
    "qwen2.5-3b": Arch("qwen2.5-3b", "qwen2", 2048, 36, 16, 2, 128, 11008, 151936, 1e-6, 1e6,
                       True, True),
    "qwen2.5-7b": Arch("qwen2.5-7b", "qwen2", 3584, 28, 28, 4, 128, 18944, 152064, 1e-6, 1e6,
                       True, False),
    # test-sized architectures (not benchmark configurations)
    "tiny-llama": Arch("tiny-llama", "llama", 128, 2, 4, 2, 32, 256, 512, 1e-5, 1e4, False, True),
    "tiny-qwen2": Arch("tiny-qwen2", "qwen2", 128, 2, 4, 2, 32, 384, 512, 1e-6, 1e6, True, True),
}


def get_arch(name: str) -> Arch:
    try:
        return ARCHITECTURES[name]
    except KeyError as exc:
        from mround_b200.exceptions import ArchitectureError

        raise ArchitectureError(
            f"unknown architecture {name!r}; known: {', '.join(sorted(ARCHITECTURES))}"
        ) from exc
