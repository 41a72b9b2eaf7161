"""CPU restatement of the reference packed refresh executor.

TEST INFRASTRUCTURE ONLY. This module is the checker for the CUDA path and the
timed CPU restatement in ``bench.py``'s reference arm. The product package never
imports it, and no product path falls back to it.

Every function restates one piece of ``yh0903/budgeted-kv-cache-repair`` (paths
below are relative to that project) or of the transformers modeling code it
drives (transformers is pinned to 4.57.6 by the reference, ``pyproject.toml:14``;
this image has 5.5.0 and the math cited below is identical in both).

Pinning: ``tests/test_oracle_golden.py`` checks these functions against
``tests/golden/*.pt``, which ``tests/golden/make_golden.py`` produced by running
the reference itself (through ``tests/golden/ref_compat.py``) on seeded tiny
models. fp32 cases agree to 1e-6; the positional correction agrees bit for bit.

Arithmetic follows the reference per operation: every tensor op runs in the
cache/model dtype with torch's CPU kernels, so each intermediate is rounded to
bf16/fp16 exactly where the reference rounds it. Attention is evaluated in fp32
from the dtype inputs and rounded once on output (SDPA semantics).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from numbers import Integral
from typing import Sequence

import torch
import torch.nn.functional as F


# --------------------------------------------------------------------------
# Token alignment: alignment.py:6-30
# --------------------------------------------------------------------------

def token_alignment(old_ids: Sequence[int], new_ids: Sequence[int]) -> dict[str, int]:
    """Common prefix/suffix of two id lists (alignment.py:6-30)."""
    old_ids, new_ids = list(old_ids), list(new_ids)
    prefix = 0
    while prefix < min(len(old_ids), len(new_ids)) and old_ids[prefix] == new_ids[prefix]:
        prefix += 1
    limit = min(len(old_ids) - prefix, len(new_ids) - prefix)
    suffix = 0
    while suffix < limit and old_ids[-1 - suffix] == new_ids[-1 - suffix]:
        suffix += 1
    return {
        "prefix": prefix,
        "suffix": suffix,
        "old_suffix_start": len(old_ids) - suffix,
        "new_suffix_start": len(new_ids) - suffix,
        "mandatory_changed_tokens": len(new_ids) - prefix - suffix,
        "position_shift": (len(new_ids) - suffix) - (len(old_ids) - suffix),
    }


# --------------------------------------------------------------------------
# Interval rules: kernels/executor.py:50-70, execution.py:14-23
# --------------------------------------------------------------------------

def validate_intervals(intervals, logical_length: int) -> tuple[tuple[int, int], ...]:
    """Sorted, disjoint, non-adjacent half-open ranges (kernels/executor.py:50-70)."""
    if not isinstance(intervals, (list, tuple)):
        raise ValueError("intervals must be a list or tuple")
    out, previous_end = [], -1
    for interval in intervals:
        if not isinstance(interval, (tuple, list)) or len(interval) != 2:
            raise ValueError("each interval must contain exactly a start and end")
        if any(isinstance(v, bool) or not isinstance(v, Integral) for v in interval):
            raise ValueError("interval bounds must be integers")
        start, end = int(interval[0]), int(interval[1])
        if not 0 <= start < end <= logical_length:
            raise ValueError("interval bounds out of range")
        if start <= previous_end:
            raise ValueError("intervals must be sorted, disjoint and non-adjacent")
        out.append((start, end))
        previous_end = end
    return tuple(out)


def positions_to_intervals(positions) -> list[tuple[int, int]]:
    """Maximal runs of sorted unique positions (execution.py:14-23)."""
    runs: list[tuple[int, int]] = []
    for p in sorted(set(int(x) for x in positions)):
        if runs and p == runs[-1][1]:
            runs[-1] = (runs[-1][0], p + 1)
        else:
            runs.append((p, p + 1))
    return runs


def plan_tiles(positions: Sequence[int], block_m: int = 16, block_n: int = 64):
    """Per query tile: unmasked key tiles and total key tiles (kernels/indexed_attention.py:75-80)."""
    full, total = [], []
    for row in range(0, len(positions), block_m):
        tile = positions[row:row + block_m]
        full.append((tile[0] + 1) // block_n)
        total.append((tile[-1] + block_n) // block_n)
    return tuple(full), tuple(total)


# --------------------------------------------------------------------------
# RoPE: transformers LlamaRotaryEmbedding (modeling_llama.py, 5.5.0 lines 92-135;
# Qwen3RotaryEmbedding is the same code) and cache.py:25-28, 47-77
# --------------------------------------------------------------------------

def default_inv_freq(theta: float, head_dim: int) -> torch.Tensor:
    """``1 / theta ** (arange(0, D, 2) / D)`` in fp32 (compute_default_rope_parameters)."""
    exponent = torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim
    return 1.0 / (theta ** exponent)


def rope_cos_sin(inv_freq: torch.Tensor, positions, dtype: torch.dtype):
    """cos/sin rows ``[P, D]`` for integer positions, fp32 math cast to ``dtype``.

    The rotary forward forms ``inv_freq @ positions`` with K=1 (one rounded fp32
    product per element), concatenates the half table twice, takes fp32 cos/sin,
    multiplies by attention_scaling (1.0 for default RoPE) and casts.
    """
    pos = torch.as_tensor(positions, dtype=torch.int64).reshape(-1).float()
    freqs = pos[:, None] * inv_freq.float()[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """Split-half rotation ``[x1, x2] -> [-x2, x1]`` (cache.py:25-28)."""
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x*cos + rotate_half(x)*sin`` with each op rounded to x's dtype."""
    return (x * cos) + (rotate_half(x) * sin)


def shifted_suffix_keys(key: torch.Tensor, shift: int, inv_freq: torch.Tensor) -> torch.Tensor:
    """Delta-RoPE of retained suffix keys ``[1, Hkv, S, D]`` (cache.py:47-77).

    A zero shift or an empty suffix returns a clone (cache.py:51-52). Every row
    rotates by the same angle ``shift * inv_freq`` (cache.py:54-60).
    """
    if not key.shape[2] or not shift:
        return key.clone()
    cos, sin = rope_cos_sin(inv_freq, [shift], key.dtype)
    return apply_rope(key, cos[0], sin[0])


def clone_layers(layers, length: int | None = None):
    """Independent copies of every layer's K/V, optionally a prefix (cache.py:31-44)."""
    out = []
    for key, value in layers:
        end = key.shape[2] if length is None else int(length)
        out.append((key[:, :, :end].clone(), value[:, :, :end].clone()))
    return out


def build_shift_cache(old_layers, old_ids, new_ids, inv_freq):
    """Shift cache with halo 0 and no changed boundary tokens (cache.py:103-144).

    Returns ``(layers, alignment)``. Each layer is ``cat(prefix, rope(K tail))``
    and ``cat(prefix, V tail)``. Changed boundary tokens need a model forward
    (cache.py:122-127) and are rejected here.
    """
    alignment = token_alignment(old_ids, new_ids)
    if alignment["mandatory_changed_tokens"]:
        raise ValueError("oracle shift cache covers deletions without changed boundary tokens")
    prefix, tail = alignment["prefix"], alignment["old_suffix_start"]
    out = []
    for key, value in old_layers:
        tail_key = shifted_suffix_keys(key[:, :, tail:], alignment["position_shift"], inv_freq)
        out.append((torch.cat((key[:, :, :prefix].clone(), tail_key), dim=2),
                    torch.cat((value[:, :, :prefix].clone(), value[:, :, tail:].clone()), dim=2)))
    return out, alignment


# --------------------------------------------------------------------------
# Decoder math: transformers LlamaRMSNorm / LlamaMLP / LlamaAttention /
# LlamaDecoderLayer (modeling_llama.py 5.5.0 lines 53-67, 163-183, 229-330)
# and Qwen3Attention q_norm/k_norm (modeling_qwen3.py 5.5.0 lines 248-268)
# --------------------------------------------------------------------------

@dataclass
class OracleModel:
    """Weights of a dense Llama/Qwen3 decoder, by transformers parameter name."""

    embed: torch.Tensor
    layers: list[dict[str, torch.Tensor]]
    heads: int
    kv_heads: int
    head_dim: int
    eps: float
    inv_freq: torch.Tensor
    qk_norm: bool

    @classmethod
    def from_state_dict(cls, state: dict, config, inv_freq: torch.Tensor | None = None) -> "OracleModel":
        """Accepts ``model.state_dict()`` of a LlamaForCausalLM/Qwen3ForCausalLM or its base model.

        ``inv_freq`` is the model's rotary buffer as stored. ``model.to(bf16)``
        casts that buffer too, and the rotary forward upcasts the rounded
        values (``self.inv_freq[None, :, None].float()``), so the buffer, not a
        fresh fp32 recomputation, defines the reference's angles.
        """
        prefix = "model." if any(k.startswith("model.") for k in state) else ""
        layers = []
        for i in range(config.num_hidden_layers):
            p = f"{prefix}layers.{i}."
            layer = {
                "in_norm": state[p + "input_layernorm.weight"],
                "q": state[p + "self_attn.q_proj.weight"],
                "k": state[p + "self_attn.k_proj.weight"],
                "v": state[p + "self_attn.v_proj.weight"],
                "o": state[p + "self_attn.o_proj.weight"],
                "post_norm": state[p + "post_attention_layernorm.weight"],
                "gate": state[p + "mlp.gate_proj.weight"],
                "up": state[p + "mlp.up_proj.weight"],
                "down": state[p + "mlp.down_proj.weight"],
            }
            if p + "self_attn.q_norm.weight" in state:
                layer["q_norm"] = state[p + "self_attn.q_norm.weight"]
                layer["k_norm"] = state[p + "self_attn.k_norm.weight"]
            layers.append(layer)
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        theta = config.rope_parameters["rope_theta"] if hasattr(config, "rope_parameters") else config.rope_theta
        return cls(
            embed=state[prefix + "embed_tokens.weight"], layers=layers,
            heads=config.num_attention_heads, kv_heads=config.num_key_value_heads,
            head_dim=head_dim, eps=config.rms_norm_eps,
            inv_freq=(default_inv_freq(float(theta), head_dim) if inv_freq is None else inv_freq).float(),
            qk_norm="q_norm" in layers[0],
        )


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """fp32 mean of squares, rsqrt, cast back, then ``weight *`` in the model dtype."""
    dtype = x.dtype
    h = x.to(torch.float32)
    variance = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(variance + eps)
    return weight * h.to(dtype)


def selected_attention(q, k, v, positions, scale: float) -> torch.Tensor:
    """Absolute-causal attention of packed queries (kernels/packed_cache.py:47-67, 203-207).

    q ``[B, Hq, D]``; k/v ``[Hkv, N, D]``; row b sees keys ``<= positions[b]``.
    GQA maps query head ``h`` to KV head ``h // (Hq/Hkv)`` (repeat_kv). fp32
    math from the dtype inputs; one rounding to q's dtype on output.
    """
    rows, heads, dim = q.shape
    kv_heads, length, _ = k.shape
    group = heads // kv_heads
    qf = q.float().permute(1, 0, 2)                               # [Hq, B, D]
    kf = k.float().repeat_interleave(group, dim=0)                # [Hq, N, D]
    vf = v.float().repeat_interleave(group, dim=0)
    scores = torch.matmul(qf, kf.transpose(-1, -2)) * scale       # [Hq, B, N]
    pos = torch.as_tensor(positions, dtype=torch.int64)
    allowed = torch.arange(length)[None, :] <= pos[:, None]
    scores = scores.masked_fill(~allowed[None], float("-inf"))
    out = torch.matmul(torch.softmax(scores, dim=-1), vf)          # [Hq, B, D]
    return out.permute(1, 0, 2).to(q.dtype)


def selected_attention_fp64(q, k, v, positions, scale: float | None = None) -> torch.Tensor:
    """Dense fp64 reference with ``[1,Hq,B,D]`` / ``[1,Hkv,N,D]`` layout.

    Restates the reference's independent kernel oracle
    (tests/test_indexed_attention.py:106-116).
    """
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    groups = q.shape[1] // k.shape[1]
    keys = k.double().repeat_interleave(groups, dim=1)
    values = v.double().repeat_interleave(groups, dim=1)
    scores = torch.matmul(q.double(), keys.transpose(-1, -2)) * scale
    absolute = torch.as_tensor(list(positions), dtype=torch.int64, device=q.device)
    allowed = torch.arange(k.shape[2], device=q.device)[None, :] <= absolute[:, None]
    scores = scores.masked_fill(~allowed[None, None], float("-inf"))
    return torch.matmul(scores.softmax(-1), values)


def packed_refresh(model: OracleModel, base_layers, ids, positions):
    """Layer-major refresh of the selected rows (kernels/packed_cache.py:225-298).

    ``base_layers``: list of ``(K, V)`` ``[1, Hkv, N, D]``; ``ids``: ``[N]`` or
    ``[1, N]`` token ids; ``positions``: sorted selected absolute rows. Returns
    new independent layers; the base is not modified. Empty support returns the
    base list itself (kernels/packed_cache.py:274-275).
    """
    positions = [int(p) for p in positions]
    if not positions:
        return base_layers
    out = clone_layers(base_layers)                              # packed_cache.py:287
    dtype = out[0][0].dtype
    pos = torch.tensor(positions, dtype=torch.int64)
    ids = torch.as_tensor(ids).reshape(-1)
    rows, heads, kv_heads, dim = len(positions), model.heads, model.kv_heads, model.head_dim
    hidden = F.embedding(ids.index_select(0, pos), model.embed)  # packed_cache.py:291
    cos, sin = rope_cos_sin(model.inv_freq, positions, dtype)   # position_ids = positions
    cos, sin = cos[:, None, :], sin[:, None, :]
    scale = dim ** -0.5
    for index, layer in enumerate(model.layers):
        residual = hidden
        x = rms_norm(hidden, layer["in_norm"], model.eps)
        q = F.linear(x, layer["q"]).view(rows, heads, dim)
        k = F.linear(x, layer["k"]).view(rows, kv_heads, dim)
        v = F.linear(x, layer["v"]).view(rows, kv_heads, dim)
        if model.qk_norm:
            q = rms_norm(q, layer["q_norm"], model.eps)
            k = rms_norm(k, layer["k_norm"], model.eps)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        key_cache, value_cache = out[index]
        key_cache.index_copy_(2, pos, k.permute(1, 0, 2).unsqueeze(0))   # packed_cache.py:189-191
        value_cache.index_copy_(2, pos, v.permute(1, 0, 2).unsqueeze(0))
        attn = selected_attention(q, key_cache[0], value_cache[0], positions, scale)
        hidden = residual + F.linear(attn.reshape(rows, heads * dim), layer["o"])
        residual = hidden
        x = rms_norm(hidden, layer["post_norm"], model.eps)
        mlp = F.linear(F.silu(F.linear(x, layer["gate"])) * F.linear(x, layer["up"]), layer["down"])
        hidden = residual + mlp
    return out


def fresh_rows(layers, positions):
    """Selected rows ``[L, 2, Hkv, B, D]`` of a cache, for row-wise comparisons."""
    pos = torch.as_tensor(list(positions), dtype=torch.int64, device=layers[0][0].device)
    return torch.stack([torch.stack((k[0].index_select(1, pos), v[0].index_select(1, pos))) for k, v in layers])


def row_cosine(actual: torch.Tensor, expected: torch.Tensor) -> torch.Tensor:
    """Cosine similarity per cache row (last dim), in fp64."""
    a, b = actual.double(), expected.double()
    num = (a * b).sum(-1)
    den = a.norm(dim=-1) * b.norm(dim=-1)
    return torch.where(den > 0, num / den.clamp_min(1e-300), torch.ones_like(num))


def causal_pairs(positions) -> int:
    """Number of (query, key) pairs the selected rows attend over."""
    return sum(int(p) + 1 for p in positions)


def rope_bytes(layers: int, kv_heads: int, rows: int, head_dim: int, elem: int = 2) -> int:
    """Algorithmic bytes of the delta-RoPE fix: read + write of every suffix K row."""
    return 2 * layers * kv_heads * rows * head_dim * elem


def attention_flops(heads: int, head_dim: int, positions, layers: int) -> float:
    """``4 * Hq * D * sum(p+1) * L`` multiply-adds x2 for QK^T and PV."""
    return 4.0 * heads * head_dim * causal_pairs(positions) * layers


__all__ = [name for name in dir() if not name.startswith("_") and name not in ("annotations", "math")]
