"""Shared test helpers: fixture models on a device, cache conversion, bit checks."""

from __future__ import annotations

from types import SimpleNamespace

import torch


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    return a.shape == b.shape and a.dtype == b.dtype and torch.equal(
        a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


def hf_config(record):
    from transformers import LlamaConfig, Qwen3Config

    c = record["config"]
    options = dict(vocab_size=c["vocab_size"], hidden_size=c["hidden_size"],
                   intermediate_size=c["intermediate_size"], num_hidden_layers=c["num_hidden_layers"],
                   num_attention_heads=c["num_attention_heads"], num_key_value_heads=c["num_key_value_heads"],
                   head_dim=c["head_dim"], rope_theta=c["rope_theta"], rms_norm_eps=c["rms_norm_eps"],
                   max_position_embeddings=4096, attention_dropout=0.0)
    if c["family"] == "llama":
        return LlamaConfig(**options)
    return Qwen3Config(**options, layer_types=["full_attention"] * c["num_hidden_layers"])


def fixture_model(record, device):
    """The fixture's model (weights and rotary buffer as recorded) on ``device``."""
    from transformers import LlamaForCausalLM, Qwen3ForCausalLM

    config = hf_config(record)
    dtype = getattr(torch, record["dtype"])
    cls = LlamaForCausalLM if record["config"]["family"] == "llama" else Qwen3ForCausalLM
    torch.manual_seed(0)
    model = cls(config).to(dtype=dtype)
    missing, unexpected = model.model.load_state_dict(record["state_dict"], strict=True), None
    model.model.rotary_emb.inv_freq = record["inv_freq"].clone()
    return model.to(device).eval()


def oracle_config(record):
    c = record["config"]
    return SimpleNamespace(num_hidden_layers=c["num_hidden_layers"], hidden_size=c["hidden_size"],
                           num_attention_heads=c["num_attention_heads"],
                           num_key_value_heads=c["num_key_value_heads"], head_dim=c["head_dim"],
                           rms_norm_eps=c["rms_norm_eps"], rope_parameters={"rope_theta": c["rope_theta"]})


def to_cache(pairs, device):
    from budgeted_kv_cache_repair_b200.cache import make_cache

    return make_cache([(k.to(device).contiguous(), v.to(device).contiguous()) for k, v in pairs])


def layers_cpu(cache):
    from budgeted_kv_cache_repair_b200.validate import cache_layers

    return [(k.detach().cpu(), v.detach().cpu()) for k, v in cache_layers(cache)]
