"""Packed selected-row refresh on the B200 (drop-in for the reference's
``packed_interval_repair``, kernels/packed_cache.py:225-298).

Same signature, validation order, error types, receipt keys and ownership
contract; the native decoder forward with per-layer ``index_copy_`` and masked
SDPA is replaced by one ``engine.refresh_rows`` call that also makes the owned
copy of the cache, layer by layer, overlapped with the refresh of earlier
layers.
"""

from __future__ import annotations

from typing import Any, Sequence

import torch

from . import _lib
from .cache import allocate_arena, arena_layers, make_cache
from .engine import model_view, refresh_rows
from .plan import IndexedPlan
from .validate import qualify_model, validate_cache, validate_intervals

# The reference's default backend names select this engine's kernels, so a
# call with default arguments (api.py:235) lands here. The reference's
# experimental Triton and Flex paths are not built: one attention path, no
# multi-backend dispatch.
ATTENTION_BACKENDS = ("sdpa", "sm100a")
WRITEBACK_BACKENDS = ("torch", "sm100a")
ENGINE = "kvr_b200/sm_100a"


def make_receipt(intervals, length: int, layer_count: int, attention_backend: str = "sdpa",
                 writeback_backend: str = "torch") -> dict[str, Any]:
    """The reference's receipt keys (kernels/packed_cache.py:259-273) plus ``engine``."""
    selected = [p for start, end in intervals for p in range(start, end)]
    return {
        "executor": "packed_interval_repair",
        "schedule": "packed_selected_rows_layer_major",
        "attention_backend": attention_backend,
        "writeback_backend": writeback_backend,
        "interval_count": len(intervals),
        "recomputed_tokens": len(selected),
        "logical_length": length,
        "layer_count": layer_count,
        "base_cache_ownership": "borrowed_immutable",
        "output_cache_ownership": "independent" if selected else "borrowed_base",
        "selected_absolute_positions": selected,
        "native_model_mutated": False,
        "numerical_contract": "separate_schedule_qualification_required",
        "engine": ENGINE,
    }


def _check_ids(edited_ids_t) -> int:
    if not isinstance(edited_ids_t, torch.Tensor) or edited_ids_t.ndim != 2 or edited_ids_t.shape[0] != 1:
        raise ValueError("edited_ids_t must be a single-batch rank-two tensor")
    if edited_ids_t.dtype not in (torch.int32, torch.int64):
        raise ValueError("edited_ids_t must contain int32 or int64 IDs")
    return int(edited_ids_t.shape[1])


def _request_ids(edited_ids_t: torch.Tensor, device: torch.device) -> torch.Tensor:
    """The ids row as the engine takes it: pinned host int64 ids as they are
    (copied once, straight into the request's staged device buffer), anything
    else as a contiguous int64 device tensor."""
    ids = edited_ids_t[0]
    if ids.device.type == "cpu" and ids.dtype == torch.int64 and ids.is_pinned() and ids.is_contiguous():
        return ids
    return _device_ids(edited_ids_t, device)


def _device_ids(edited_ids_t: torch.Tensor, device: torch.device) -> torch.Tensor:
    ids = edited_ids_t[0]
    if ids.device != device:
        if ids.device.type == "cpu" and not ids.is_pinned():
            from .staging import upload_int64

            return upload_int64(ids, device)
        ids = ids.to(device, non_blocking=True)
    if ids.dtype != torch.int64:
        ids = ids.to(torch.int64)
    return ids.contiguous()


def _base_and_dtype(shim, layers, device):
    model = shim.generator
    base = shim._base_transformer(model)
    dtype = layers[0][0].dtype
    if dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("the B200 packed executor computes in bfloat16 or float16")
    qualify_model(model, base, len(layers), device, dtype)
    return base


def _check_plan(plan, selected, length: int) -> None:
    if not isinstance(plan, IndexedPlan) or tuple(plan.positions) != selected or plan.logical_length != length:
        raise ValueError("supplied IndexedPlan must match exact selected positions and cache length")


def refresh_owned_layers(shim: Any, layers, edited_ids_t: torch.Tensor, intervals, plan: IndexedPlan | None = None):
    """Refresh ``intervals`` in place in caller-owned layer tensors (no copy, no receipt)."""
    length = _check_ids(edited_ids_t)
    intervals = validate_intervals(intervals, length)
    selected = tuple(p for start, end in intervals for p in range(start, end))
    if not selected:
        return
    device = layers[0][0].device
    if device.type != "cuda":
        raise ValueError("the B200 packed executor requires CUDA tensors")
    base = _base_and_dtype(shim, layers, device)
    if plan is not None:
        _check_plan(plan, selected, length)
    with torch.cuda.device(device):
        ids = _request_ids(edited_ids_t, device)
        # The validated host positions go to the device with the request's
        # other inputs (one pinned copy into the staged buffer).
        refresh_rows(model_view(base), layers, ids, selected, selected[-1], length)


@torch.no_grad()
def packed_interval_repair(
    shim: Any, base_cache: Any, edited_ids_t: torch.Tensor,
    intervals: Sequence[tuple[int, int]], *,
    attention_backend: str = "sdpa", writeback_backend: str = "torch",
    plan: Any = None,
) -> tuple[Any, dict[str, Any]]:
    """Recompute sorted selected rows in one layer-major pass on the B200.

    ``plan`` optionally supplies a reusable host ``IndexedPlan`` for exactly
    these intervals and this logical length. Returns ``(cache, receipt)``:
    a new ``DynamicCache`` owning its storage, bit-identical to ``base_cache``
    outside the selected rows, or ``base_cache`` itself for an empty support.
    ``base_cache`` is never modified, including on failure.
    """
    if attention_backend not in ATTENTION_BACKENDS:
        raise ValueError("attention_backend must be 'sdpa' (default) or 'sm100a'; "
                         "the Triton/Flex prototypes are not part of the B200 engine")
    if writeback_backend not in WRITEBACK_BACKENDS:
        raise ValueError("writeback_backend must be 'torch' (default) or 'sm100a'")
    length = _check_ids(edited_ids_t)
    layers = validate_cache(base_cache, length)
    intervals = validate_intervals(intervals, length)
    selected = tuple(p for start, end in intervals for p in range(start, end))
    if plan is not None:
        _check_plan(plan, selected, length)
    receipt = make_receipt(intervals, length, len(layers), attention_backend, writeback_backend)
    if not selected:
        return base_cache, receipt
    device = layers[0][0].device
    if device.type != "cuda" or edited_ids_t.device.type not in ("cpu", "cuda"):
        raise ValueError("the B200 packed executor requires a CUDA cache (there is no CPU path)")
    if any(k.device != device or v.device != device for k, v in layers):
        raise ValueError("packed executor requires all cache layers on the request device")
    base = _base_and_dtype(shim, layers, device)
    view = model_view(base)
    if layers[0][0].shape[1] != view.kv_heads or layers[0][0].shape[3] != view.head_dim:
        raise ValueError("cache head geometry does not match the model")
    _lib.load()
    # The selected positions come from validated intervals (sorted, disjoint,
    # inside the cache), so they already are what an IndexedPlan of them would
    # hold; the engine needs no tile metadata, so none is built here.
    with torch.cuda.device(device):
        ids = _request_ids(edited_ids_t, device)
        # The ownership copy (kernels/packed_cache.py:287) runs inside the
        # refresh call, each layer's copy overlapping earlier layers' work; the
        # validated host positions reach the device there too.
        # The kernels take the output block's layer addresses; its per-layer
        # views are made after the launch, while the device works.
        arena = allocate_arena(len(layers), view.kv_heads, length, view.head_dim, layers[0][0].dtype, device)
        refresh_rows(view, arena, ids, selected, selected[-1], length, sources=layers)
    return make_cache(arena_layers(arena)), receipt
