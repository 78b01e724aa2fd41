"""Local Hugging Face checkpoint loading (CPU): a tiny Llama/Qwen2 checkpoint
written in the HF layout (config.json, sharded safetensors with an index) is
read back tensor for tensor, and what the reference refuses is refused
(mround/pipeline/loader.py:245-254), as is what the device path does not
implement."""

from __future__ import annotations

import json

import pytest
import torch

from mround_b200.exceptions import ArchitectureError
from mround_b200.formats.safetensors_io import write_safetensors
from mround_b200.pipeline.arch import get_arch
from mround_b200.pipeline.loader import CheckpointModel
from mround_b200.pipeline.model import SyntheticModel


def write_checkpoint(tmp, arch_name="tiny-qwen2", seed=3, *, shards=2, edit_config=None,
                     linear_dtype=torch.bfloat16, extra=None):
    model = SyntheticModel(get_arch(arch_name), seed=seed)
    tensors = {"model.embed_tokens.weight": model.embed_tokens()}
    for i in range(model.arch.layers):
        p = model.block(i)
        name = model.block_name(i)
        for path, w in p.linears.items():
            tensors[f"{name}.{path}.weight"] = w.to(linear_dtype)
        for path, b in p.biases.items():
            tensors[f"{name}.{path}.bias"] = b
        tensors[f"{name}.input_layernorm.weight"] = p.input_norm
        tensors[f"{name}.post_attention_layernorm.weight"] = p.post_norm
    tensors["model.norm.weight"] = model.final_norm()
    if not model.arch.tied:
        tensors["lm_head.weight"] = model.lm_head()
    tensors.update(extra or {})
    names = list(tensors)
    weight_map = {}
    for s in range(shards):
        part = names[s::shards]
        fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        write_safetensors(tmp / fname, {n: tensors[n] for n in part}, metadata={"format": "pt"})
        weight_map.update({n: fname for n in part})
    (tmp / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    config = model.config()
    config["architectures"] = ["Qwen2ForCausalLM" if model.arch.family == "qwen2"
                               else "LlamaForCausalLM"]
    if edit_config:
        edit_config(config)
    (tmp / "config.json").write_text(json.dumps(config))
    return model


@pytest.mark.parametrize("arch_name", ["tiny-qwen2", "tiny-llama"])
def test_checkpoint_round_trip(tmp_path, arch_name):
    model = write_checkpoint(tmp_path, arch_name)
    ck = CheckpointModel(tmp_path)
    a, b = ck.arch, model.arch
    for field in ("family", "hidden", "layers", "heads", "kv_heads", "head_dim", "intermediate",
                  "vocab", "rms_eps", "rope_theta", "qkv_bias", "tied"):
        assert getattr(a, field) == getattr(b, field), field
    for i in range(a.layers):
        got, want = ck.block(i), model.block(i)
        for path in want.linears:
            assert torch.equal(got.linears[path].view(torch.int16),
                               want.linears[path].view(torch.int16))
        assert set(got.biases) == set(want.biases)
        for path in want.biases:
            assert torch.equal(got.biases[path], want.biases[path])
        assert torch.equal(got.input_norm, want.input_norm)
    assert torch.equal(ck.embed_tokens(), model.embed_tokens())
    assert torch.equal(ck.lm_head(), model.lm_head())
    assert ck.config()["model_type"] == b.family


def test_load_model_routes_directories(tmp_path):
    from mround_b200.api import load_model

    write_checkpoint(tmp_path)
    assert isinstance(load_model(str(tmp_path)), CheckpointModel)
    with pytest.raises(ArchitectureError):
        load_model(str(tmp_path / "missing"))


@pytest.mark.parametrize("edit,msg", [
    (lambda c: c.update(quantization={"bits": 4, "group_size": 64}), "already quantized"),
    (lambda c: c.update(model_type="gemma"), "not supported"),
    (lambda c: c.update(rope_scaling={"type": "llama3", "factor": 8.0}), "rope_scaling"),
    (lambda c: (c.pop("rope_theta", None),
                c.update(rope_parameters={"rope_type": "yarn", "rope_theta": 1e6,
                                          "factor": 4.0})), "rope_type"),
    (lambda c: c.update(use_sliding_window=True, sliding_window=1024), "sliding_window"),
    (lambda c: c.update(mlp_bias=True), "mlp_bias"),
])
def test_refusals(tmp_path, edit, msg):
    write_checkpoint(tmp_path, edit_config=edit)
    with pytest.raises(ArchitectureError, match=msg):
        CheckpointModel(tmp_path)


def test_llama_attention_bias_refused(tmp_path):
    """Llama's attention_bias puts a bias on o_proj too, which the block would drop."""
    write_checkpoint(tmp_path, "tiny-llama", edit_config=lambda c: c.update(attention_bias=True))
    with pytest.raises(ArchitectureError, match="o_proj"):
        CheckpointModel(tmp_path)


@pytest.mark.parametrize("path", ["self_attn.o_proj", "mlp.down_proj"])
def test_unapplied_bias_tensors_refused(tmp_path, path):
    """A bias tensor the block does not apply is refused even when the
    configuration does not declare it."""
    rows = get_arch("tiny-llama").linear_shapes()[path][0]
    write_checkpoint(tmp_path, "tiny-llama",
                     extra={f"model.layers.0.{path}.bias": torch.zeros(rows, dtype=torch.bfloat16)})
    ck = CheckpointModel(tmp_path)
    with pytest.raises(ArchitectureError, match="bias"):
        ck.block(0)


def test_rope_theta_from_rope_parameters(tmp_path):
    """transformers >= 5 configs carry the theta under ``rope_parameters``."""
    def edit(c):
        c.pop("rope_theta", None)
        c["rope_parameters"] = {"rope_type": "default", "rope_theta": 123456.0}

    write_checkpoint(tmp_path, edit_config=edit)
    assert CheckpointModel(tmp_path).arch.rope_theta == 123456.0


def test_non_bf16_linears_refused(tmp_path):
    write_checkpoint(tmp_path, linear_dtype=torch.float32)
    ck = CheckpointModel(tmp_path)
    with pytest.raises(ArchitectureError, match="bf16"):
        ck.block(0)


def test_cli_dry_run_on_checkpoint(tmp_path, capsys):
    from mround_b200.cli.main import main

    write_checkpoint(tmp_path)
    assert main(["quantize", str(tmp_path), "-o", str(tmp_path / "out"), "--bits", "2",
                 "--asym", "--dry-run"]) == 0


@pytest.mark.parametrize("family", ["qwen2", "llama"])
def test_reads_a_checkpoint_written_by_transformers(tmp_path, family):
    """A tiny model saved by transformers' own ``save_pretrained`` (bf16,
    safetensors) loads here with every tensor equal and the architecture read
    from its config.json."""
    transformers = pytest.importorskip("transformers")
    if family == "qwen2":
        cfg = transformers.Qwen2Config(hidden_size=64, intermediate_size=160, num_hidden_layers=2,
                                       num_attention_heads=4, num_key_value_heads=2,
                                       vocab_size=300, rms_norm_eps=1e-6,
                                       tie_word_embeddings=True, max_position_embeddings=256,
                                       rope_parameters={"rope_type": "default",
                                                        "rope_theta": 5.0e5})
        lm = transformers.Qwen2ForCausalLM(cfg)
    else:
        cfg = transformers.LlamaConfig(hidden_size=64, intermediate_size=160, num_hidden_layers=2,
                                       num_attention_heads=4, num_key_value_heads=2,
                                       vocab_size=300, rms_norm_eps=1e-5,
                                       tie_word_embeddings=False, max_position_embeddings=256,
                                       rope_parameters={"rope_type": "default",
                                                        "rope_theta": 5.0e5})
        lm = transformers.LlamaForCausalLM(cfg)
    lm = lm.to(torch.bfloat16)
    lm.save_pretrained(tmp_path, safe_serialization=True)
    ck = CheckpointModel(tmp_path)
    arch = ck.arch
    assert (arch.family, arch.hidden, arch.layers, arch.heads, arch.kv_heads) == (family, 64, 2, 4, 2)
    assert arch.head_dim == 16 and arch.intermediate == 160 and arch.vocab == 300
    assert arch.qkv_bias == (family == "qwen2") and arch.tied == (family == "qwen2")
    assert arch.rope_theta == 5.0e5 and arch.rms_eps == cfg.rms_norm_eps
    state = lm.state_dict()
    assert torch.equal(ck.embed_tokens().to(torch.bfloat16), state["model.embed_tokens.weight"])
    assert torch.equal(ck.final_norm().to(torch.bfloat16), state["model.norm.weight"])
    if not arch.tied:
        assert torch.equal(ck.lm_head().to(torch.bfloat16), state["lm_head.weight"])
    for i in range(2):
        p = ck.block(i)
        for path, w in p.linears.items():
            assert torch.equal(w, state[f"model.layers.{i}.{path}.weight"]), path
        for path, b in p.biases.items():
            assert torch.equal(b.to(torch.bfloat16), state[f"model.layers.{i}.{path}.bias"]), path
        assert torch.equal(p.input_norm.to(torch.bfloat16),
                           state[f"model.layers.{i}.input_layernorm.weight"])
