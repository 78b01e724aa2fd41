"""The oracle's decoder block against Hugging Face transformers' layer.

The reference runs mlx-lm's Llama/Qwen2 decoder layer (mlx-lm is not
installed here); mlx-lm's layers implement the same architecture definitions
as transformers' ``LlamaDecoderLayer`` / ``Qwen2DecoderLayer``.  Loading one
synthetic block's weights into the transformers layer (eager attention, an
additive causal mask, the model's own rotary embedding) and into
``oracle.block_tuner.OracleBlock`` must give the same output to float32
rounding: RMSNorm placement and epsilon, the rotate-half RoPE with the
architecture's theta, grouped-query attention, Qwen2's q/k/v biases and the
SwiGLU MLP all agree.  This pins the block the device path is checked against
to an independent implementation.
"""

from __future__ import annotations

import pytest
import torch

from mround_b200.pipeline.arch import get_arch
from mround_b200.pipeline.model import SyntheticModel
from oracle.block_tuner import LINEARS, OracleBlock

transformers = pytest.importorskip("transformers")


def _hf_layer(arch, params):
    if arch.family == "qwen2":
        from transformers import Qwen2Config as Config
        from transformers.models.qwen2 import modeling_qwen2 as mod

        layer_cls, rope_cls = mod.Qwen2DecoderLayer, mod.Qwen2RotaryEmbedding
        extra = {}
    else:
        from transformers import LlamaConfig as Config
        from transformers.models.llama import modeling_llama as mod

        layer_cls, rope_cls = mod.LlamaDecoderLayer, mod.LlamaRotaryEmbedding
        extra = {"attention_bias": False, "mlp_bias": False, "head_dim": arch.head_dim}
    cfg = Config(hidden_size=arch.hidden, intermediate_size=arch.intermediate,
                 num_attention_heads=arch.heads, num_key_value_heads=arch.kv_heads,
                 rms_norm_eps=arch.rms_eps, vocab_size=arch.vocab, max_position_embeddings=4096,
                 rope_parameters={"rope_type": "default", "rope_theta": arch.rope_theta}, **extra)
    cfg._attn_implementation = "eager"
    layer = layer_cls(cfg, layer_idx=0).eval()
    state = {f"{p}.weight": params.linears[p].float() for p in LINEARS}
    state.update({f"{p}.bias": b.float() for p, b in params.biases.items()})
    state["input_layernorm.weight"] = params.input_norm.float()
    state["post_attention_layernorm.weight"] = params.post_norm.float()
    missing, unexpected = layer.load_state_dict(state, strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    return layer, rope_cls(cfg)


@pytest.mark.parametrize("name", ["tiny-qwen2", "tiny-llama"])
def test_oracle_block_equals_transformers_layer(name):
    arch = get_arch(name)
    params = SyntheticModel(arch, seed=3).block(0)
    oracle = OracleBlock(arch, params, {p: 4 for p in LINEARS}, 32)
    layer, rope = _hf_layer(arch, params)
    g = torch.Generator().manual_seed(7)
    b, s = 2, 96
    x = torch.randn(b, s, arch.hidden, generator=g) * 0.5
    positions = torch.arange(s)[None].expand(b, s)
    cos, sin = rope(x, positions)
    mask = torch.full((s, s), torch.finfo(torch.float32).min).triu(1)[None, None].expand(b, 1, s, s)
    with torch.no_grad():
        out = layer(x, attention_mask=mask, position_embeddings=(cos, sin))
        out = out[0] if isinstance(out, tuple) else out
        ref = oracle.forward(x)
    assert ((out - ref).abs().max() / ref.abs().max()).item() < 1e-6


@pytest.mark.parametrize("name", ["tiny-qwen2", "tiny-llama"])
def test_oracle_causal_lm_equals_transformers_model(name):
    """The whole-model forward the DeltaLoss scoring differentiates (embedding,
    every block, the final norm, the tied LM head) against transformers'
    causal-LM model holding the same synthetic weights."""
    from oracle.block_tuner import rms_norm

    arch = get_arch(name)
    model = SyntheticModel(arch, seed=5)
    if arch.family == "qwen2":
        from transformers import Qwen2Config as Config
        from transformers import Qwen2ForCausalLM as LM

        extra = {}
    else:
        from transformers import LlamaConfig as Config
        from transformers import LlamaForCausalLM as LM

        extra = {"attention_bias": False, "mlp_bias": False, "head_dim": arch.head_dim}
    cfg = Config(hidden_size=arch.hidden, intermediate_size=arch.intermediate,
                 num_attention_heads=arch.heads, num_key_value_heads=arch.kv_heads,
                 num_hidden_layers=arch.layers, rms_norm_eps=arch.rms_eps, vocab_size=arch.vocab,
                 max_position_embeddings=4096, tie_word_embeddings=arch.tied,
                 rope_parameters={"rope_type": "default", "rope_theta": arch.rope_theta}, **extra)
    cfg._attn_implementation = "eager"
    lm = LM(cfg).eval()
    state = {"model.embed_tokens.weight": model.embed_tokens().float(),
             "model.norm.weight": model.final_norm().float()}
    if not arch.tied:
        state["lm_head.weight"] = model.lm_head().float()
    blocks = []
    for i in range(arch.layers):
        params = model.block(i)
        blocks.append(OracleBlock(arch, params, {p: 4 for p in LINEARS}, 32))
        state.update({f"model.layers.{i}.{p}.weight": params.linears[p].float() for p in LINEARS})
        state.update({f"model.layers.{i}.{p}.bias": b.float() for p, b in params.biases.items()})
        state[f"model.layers.{i}.input_layernorm.weight"] = params.input_norm.float()
        state[f"model.layers.{i}.post_attention_layernorm.weight"] = params.post_norm.float()
    missing, unexpected = lm.load_state_dict(state, strict=False)
    assert not unexpected, unexpected
    assert set(missing) <= {"lm_head.weight"}, missing  # tied to the embedding
    g = torch.Generator().manual_seed(11)
    tokens = torch.randint(0, arch.vocab, (2, 40), generator=g)
    with torch.no_grad():
        logits = lm(input_ids=tokens).logits
        x = model.embed_tokens().float()[tokens]
        for blk in blocks:
            x = blk.forward(x)
        head = model.embed_tokens().float() if arch.tied else model.lm_head().float()
        ref = rms_norm(x, model.final_norm().float(), arch.rms_eps) @ head.t()
    assert ((logits - ref).abs().max() / ref.abs().max()).item() < 1e-5
