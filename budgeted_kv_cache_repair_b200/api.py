"""Public repair interface (api.py of the reference, lines 22-244).

``repair_after_deletion`` keeps the reference's signature, validation, budget
rule and result type; positional correction and the packed refresh run on the
B200 kernels. Support selection (semantic units + frozen-embedding relevance,
semantic_units.py / scoring.py) is ``selection.sur_selector``: host-side units
and allocation, relevance scores from one CUDA kernel; callers may pass any
``selector`` with the same signature instead.

When the API owns the shifted cache (it does: the caller never sees it), the
packed refresh writes into that cache in place instead of cloning it, which
removes one full cache copy per request; the caller's ``old_cache`` is still
never modified.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Callable

import torch

from .cache import OperatorShim, build_halo_cache
from .packed import make_receipt, refresh_owned_layers
from .selection import sur_selector
from .validate import cache_layers, check_model_arithmetic


@dataclass(frozen=True)
class Selection:
    """Selected absolute positions in the edited prompt, with half-open intervals (api.py:22-31)."""

    positions: tuple[int, ...]
    intervals: tuple[tuple[int, int], ...]
    suffix_start: int
    suffix_tokens: int
    budget_tokens: int
    metadata: dict[str, Any]


@dataclass(frozen=True)
class RepairResult:
    """A repaired cache and the edited prompt it represents (api.py:34-42)."""

    cache: Any
    edited_text: str
    input_ids: torch.Tensor
    selection: Selection
    metadata: dict[str, Any]


def _check_budget(budget_percent: float) -> float:
    if isinstance(budget_percent, bool):
        raise ValueError("budget_percent must be a number between 0 and 100")
    value = float(budget_percent)
    if not math.isfinite(value) or not 0.0 <= value <= 100.0:
        raise ValueError("budget_percent must be finite and between 0 and 100")
    return value


def _encode(model: Any, tokenizer: Any, text: str) -> torch.Tensor:
    ids = tokenizer(text, add_special_tokens=False, return_tensors="pt")["input_ids"]
    if not isinstance(ids, torch.Tensor) or ids.ndim != 2 or ids.shape[0] != 1:
        raise ValueError("tokenizer must return input_ids with shape [1, tokens]")
    device = model.get_input_embeddings().weight.device
    return ids.to(device=device, dtype=torch.long)


def positions_to_intervals(positions) -> list[tuple[int, int]]:
    """Coalesce sorted unique positions into maximal runs (execution.py:14-23)."""
    intervals: list[tuple[int, int]] = []
    for position in sorted(set(int(p) for p in positions)):
        if intervals and position == intervals[-1][1]:
            intervals[-1] = (intervals[-1][0], position + 1)
        else:
            intervals.append((position, position + 1))
    return intervals


def budget_tokens(suffix_tokens: int, budget_percent: float) -> int:
    """``min(S, ceil(S * percent / 100))`` (api.py:76-77)."""
    return min(suffix_tokens, math.ceil(suffix_tokens * budget_percent / 100.0))


def _select_encoded(model, tokenizer, text, query, ids, suffix_start, budget_percent,
                    selector: Callable | None = None) -> Selection:
    if isinstance(suffix_start, bool) or not isinstance(suffix_start, int):
        raise ValueError("suffix_start must be an integer token position")
    length = int(ids.shape[1])
    if not 0 <= suffix_start <= length:
        raise ValueError("suffix_start must lie inside the edited prompt")
    suffix_tokens = length - suffix_start
    budget = budget_tokens(suffix_tokens, budget_percent)
    metadata: dict[str, Any] = {"budget_percent": budget_percent}
    if budget == 0:
        positions: list[int] = []
        metadata["selection"] = "shift_only"
    elif budget == suffix_tokens:
        positions = list(range(suffix_start, length))
        metadata["selection"] = "full_suffix"
    else:
        chosen = selector or sur_selector
        picked = chosen(model, tokenizer, text, query, ids, suffix_start, budget_percent)
        positions = list(picked.positions if hasattr(picked, "positions") else picked)
        metadata.update(dict(getattr(picked, "metadata", {}) or {}))
        metadata.setdefault("selection", "external")
    if len(positions) != budget or any(not suffix_start <= p < length for p in positions) \
            or len(set(positions)) != len(positions):
        raise RuntimeError("selected support violates the suffix budget")
    positions = sorted(int(p) for p in positions)
    return Selection(tuple(positions), tuple(positions_to_intervals(positions)), suffix_start,
                     suffix_tokens, budget, metadata)


@torch.no_grad()
def select_support(model: Any, tokenizer: Any, edited_text: str, query: str, *, suffix_start: int,
                   budget_percent: float = 5.0, selector: Callable | None = None) -> Selection:
    """Allocate ``ceil(budget_percent / 100 * suffix_tokens)`` positions (api.py:113-132)."""
    budget_percent = _check_budget(budget_percent)
    ids = _encode(model, tokenizer, edited_text)
    return _select_encoded(model, tokenizer, edited_text, query, ids, suffix_start, budget_percent, selector)


def _check_model(model: Any) -> None:
    from transformers import LlamaForCausalLM, LlamaModel, Qwen3ForCausalLM, Qwen3Model

    base = getattr(model, "base_model", None)
    if (type(model), type(base)) not in {(LlamaForCausalLM, LlamaModel), (Qwen3ForCausalLM, Qwen3Model)}:
        raise ValueError("repair_after_deletion supports native dense Llama and Qwen3 models")
    if any(module.training for module in model.modules()):
        raise ValueError("call model.eval() before repairing its cache")
    check_model_arithmetic(model.config, base, "repair")
    device = model.get_input_embeddings().weight.device
    if device.type != "cuda" or any(p.device != device for p in model.parameters()):
        raise ValueError("repair on the B200 engine requires one CUDA device holding the whole model")
    if any(getattr(module, "_hf_hook", None) is not None for module in model.modules()):
        raise ValueError("repair does not support dispatch or offload hooks")
    if any("forward" in module.__dict__ for module in model.modules()):
        raise ValueError("repair does not support per-instance forward overrides")
    if getattr(model, "is_quantized", False):
        raise ValueError("repair does not support quantized models")
    if any(p.dtype not in (torch.bfloat16, torch.float16) for p in base.parameters()):
        raise ValueError("repair on the B200 engine requires a bfloat16 or float16 model")


@torch.no_grad()
def repair_after_deletion(model: Any, tokenizer: Any, old_cache: Any, original_text: str, *,
                          delete_span: tuple[int, int], query: str, budget_percent: float = 5.0,
                          executor: str = "packed", selector: Callable | None = None) -> RepairResult:
    """Delete a character span, correct positions, and refresh selected suffix KV (api.py:169-244).

    ``old_cache`` must come from an unpadded batch-one prefill of exactly
    ``tokenizer(original_text, add_special_tokens=False)``; it is not modified.
    Only ``executor="packed"`` runs on this engine.
    """
    budget_percent = _check_budget(budget_percent)
    if executor not in ("packed", "sequential"):
        raise ValueError("executor must be 'packed' or 'sequential'")
    if executor != "packed":
        raise ValueError("the B200 engine implements the packed executor; use the reference for 'sequential'")
    if (not isinstance(delete_span, (tuple, list)) or len(delete_span) != 2
            or any(isinstance(v, bool) or not isinstance(v, int) for v in delete_span)):
        raise ValueError("delete_span must contain two integer character offsets")
    start, end = delete_span
    if not 0 <= start < end <= len(original_text):
        raise ValueError("delete_span must be a nonempty half-open span in original_text")
    _check_model(model)
    old_ids = _encode(model, tokenizer, original_text)
    old_length = int(old_ids.shape[1])
    layers = cache_layers(old_cache)
    if not old_length or len(layers) != model.config.num_hidden_layers:
        raise ValueError("old_cache must contain every model layer for a nonempty prompt")
    for key, value in layers:
        if key.ndim != 4 or key.shape != value.shape or key.shape[0] != 1 or key.shape[2] != old_length:
            raise ValueError("old_cache shape does not match the batch-one original prompt")
        if key.device != old_ids.device or value.device != old_ids.device:
            raise ValueError("cache and model must be on the same device")
        if key.dtype != value.dtype or key.dtype != model.get_input_embeddings().weight.dtype:
            raise ValueError("old_cache must hold K/V in the model's dtype")
    edited_text = original_text[:start] + original_text[end:]
    edited_ids = _encode(model, tokenizer, edited_text)
    shim = OperatorShim(model, tokenizer)
    shifted_cache, alignment = build_halo_cache(shim, old_cache, old_ids, edited_ids, halo_tokens=0)
    selection = _select_encoded(model, tokenizer, edited_text, query, edited_ids,
                                int(alignment["new_suffix_start"]), budget_percent, selector)
    intervals = list(selection.intervals)
    # The shifted cache is private to this call: refresh it in place (no clone).
    layers = cache_layers(shifted_cache)
    execution = make_receipt(intervals, int(edited_ids.shape[1]), len(layers))
    execution["output_cache_ownership"] = "independent"   # new storage, never the caller's old_cache
    execution["output_storage"] = "shift_cache_refreshed_in_place"
    refresh_owned_layers(shim, layers, edited_ids, intervals)
    return RepairResult(cache=shifted_cache, edited_text=edited_text, input_ids=edited_ids,
                        selection=selection,
                        metadata={"alignment": alignment, "execution": execution, "executor": executor})
