"""Cache operators of the repair path on the B200: ownership copy, delta-RoPE
positional correction and the shift cache.

Mirrors cache.py of the reference (OperatorShim 13-22, rotate_half 25-28,
clone_cache 31-44, shifted_suffix_keys 47-77, build_halo_cache 103-144,
merge_intervals 195-204) with the per-layer eager loops replaced by one
multi-layer kernel each. Inputs are never modified; outputs own new storage.
"""

from __future__ import annotations

import operator
from itertools import repeat
from typing import Any

import torch

from . import _lib
from .alignment import token_alignment
from .validate import cache_layers, kv_strides, require_cuda_tensors


class OperatorShim:
    """The small model surface the repair operators use (cache.py:13-22)."""

    def __init__(self, model: Any, tokenizer: Any = None) -> None:
        self.generator = model
        self.tokenizer = tokenizer

    @staticmethod
    def _base_transformer(model: Any) -> Any:
        return getattr(model, "base_model", model)


def rotate_half(value: torch.Tensor) -> torch.Tensor:
    """Split-half rotation ``[x1, x2] -> [-x2, x1]`` (cache.py:25-28)."""
    left = value[..., : value.shape[-1] // 2]
    right = value[..., value.shape[-1] // 2:]
    return torch.cat((-right, left), dim=-1)


def make_cache(pairs) -> Any:
    """A transformers ``DynamicCache`` whose layers hold exactly these tensors.

    ``DynamicCache.update`` would ``torch.cat`` each tensor onto an empty one
    (a full copy); setting the layer state directly keeps the storage the
    kernels wrote, as the reference's ``_PackedLayer`` does
    (kernels/packed_cache.py:166-174).
    """
    from transformers.cache_utils import DynamicCache, DynamicLayer

    cache = DynamicCache()
    layers = []
    for key, value in pairs:
        layer = DynamicLayer()
        layer.keys, layer.values = key, value
        layer.dtype, layer.device = key.dtype, key.device
        layer.is_initialized = True
        layers.append(layer)
    cache.layers = layers
    return cache


def _check_kv_layout(tensors, what):
    for t in tensors:
        if t.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f"{what}: the B200 kernels take bfloat16 or float16 caches")
        if t.ndim != 4 or t.shape[0] != 1:
            raise ValueError(f"{what}: cache tensors must be [1, heads, tokens, head_dim]")
        if t.shape[3] % 8 or (t.stride(3) != 1 and t.shape[3] > 1):
            raise ValueError(f"{what}: head_dim must be a multiple of 8 with unit stride")
        if t.data_ptr() % 16 or t.stride(1) % 8 or t.stride(2) % 8:
            raise ValueError(f"{what}: cache rows must be 16-byte aligned")


def _uniform_strides(tensors, what):
    strides = {kv_strides(t) for t in tensors}
    if len(strides) != 1:
        raise ValueError(f"{what}: every layer must share one (head, row) stride pair")
    return strides.pop()


def allocate_arena(count: int, heads: int, rows: int, dim: int, dtype, device) -> torch.Tensor:
    """One contiguous ``[2 * count, 1, heads, rows, dim]`` block for ``count``
    ``(K, V)`` pairs (K of layer l at index 2l, V at 2l + 1): a request costs
    one allocator call instead of two per layer."""
    return torch.empty((count * 2, 1, heads, rows, dim), dtype=dtype, device=device)


def arena_layers(arena: torch.Tensor):
    """The ``(K, V)`` pairs of ``[1, heads, rows, dim]`` that an arena holds, as
    views of it; the block is released once no view is referenced any more."""
    views = arena.unbind(0)
    return [(views[2 * i], views[2 * i + 1]) for i in range(len(views) // 2)]


def allocate_layers(count: int, heads: int, rows: int, dim: int, dtype, device):
    """``count`` new ``(K, V)`` pairs of ``[1, heads, rows, dim]``, contiguous
    views of one allocation (``allocate_arena``)."""
    return arena_layers(allocate_arena(count, heads, rows, dim, dtype, device))


_dtype_of = operator.attrgetter("dtype")
_device_of = operator.attrgetter("device")


def uniform_layout(pairs, what: str):
    """Check every K/V tensor against the first one (CUDA, bf16/fp16, shape,
    strides, 16-byte rows) and return ``(heads, rows, dim, dtype, device,
    head_stride, row_stride)``."""
    first = pairs[0][0]
    require_cuda_tensors([first], what)
    _check_kv_layout([first], what)
    shape, stride, dtype, device = first.shape, first.stride(), first.dtype, first.device
    tensors = [t for pair in pairs for t in pair]
    # One C-level pass per property over all tensors; a mismatch, a
    # misaligned row or a non-tensor takes the loop below, which names it.
    try:
        fast = (set(map(type, tensors)) == {type(first)} and set(map(torch.Tensor.size, tensors)) == {shape}
                and set(map(torch.Tensor.stride, tensors)) == {stride}
                and set(map(_dtype_of, tensors)) == {dtype} and set(map(_device_of, tensors)) == {device}
                and not any(map(operator.mod, map(torch.Tensor.data_ptr, tensors), repeat(16))))
    except (TypeError, AttributeError):
        fast = False
    if not fast:
        for t in tensors:
            if t.shape != shape or t.stride() != stride or t.dtype != dtype or t.device != device:
                raise ValueError(f"{what}: every layer must share one shape, stride pair, dtype and device")
            if t.data_ptr() % 16:
                raise ValueError(f"{what}: cache rows must be 16-byte aligned")
    return shape[1], shape[2], shape[3], dtype, device, stride[1], stride[2]


def copy_layers(pairs, length: int | None = None):
    """Independent copies of every layer's K/V (prefix ``length`` if given) in one launch."""
    if not pairs:
        return []
    if len(pairs) * 2 > _lib.MAX_LAYER_TENSORS:
        raise ValueError("clone_cache: more layers than one launch takes")
    heads, rows, dim, dtype, device, src_hs, src_rs = uniform_layout(pairs, "clone_cache")
    rows = rows if length is None else int(length)
    outs = allocate_layers(len(pairs), heads, rows, dim, dtype, device)
    if rows:
        from .engine import kernel_timer

        timer = kernel_timer()
        token = timer.start("copy_layers") if timer else None
        lib = _lib.load()
        src = _lib.ptr_array([t for pair in pairs for t in pair])
        dst = _lib.ptr_array([t for pair in outs for t in pair])
        _lib.check(lib.kvr_copy_layers(src, dst, len(pairs) * 2, heads, rows, dim, src_hs, src_rs, rows * dim, dim,
                                       _lib.dtype_code(dtype), _lib.stream_handle(device)), "copy_layers")
        if token:
            timer.stop(token)
    return outs


def clone_cache(cache: Any, length: int | None = None):
    """Clone all layers, optionally only a prefix; never alias storage (cache.py:31-44)."""
    pairs = cache_layers(cache)
    if length is not None and (int(length) < 0 or (pairs and int(length) > pairs[0][0].shape[2])):
        raise ValueError("prefix length is outside the cache")
    return make_cache(copy_layers(pairs, length))


def _shift_table(model: Any, key: torch.Tensor, shift: int) -> torch.Tensor:
    """``[cos; sin]`` (2*D elements, key dtype) for one shift, from the model's
    own rotary module exactly as shifted_suffix_keys obtains it (cache.py:53-66)."""
    base = model._base_transformer(model.generator)
    positions = torch.full((1, 1), int(shift), dtype=torch.long, device=key.device)
    cos, sin = base.rotary_emb(key, positions)
    cos = cos.reshape(-1).to(device=key.device, dtype=key.dtype)
    sin = sin.reshape(-1).to(device=key.device, dtype=key.dtype)
    if cos.numel() != key.shape[-1]:
        raise ValueError("partial rotary embeddings are outside the supported model families")
    return torch.cat((cos, sin)).contiguous()


def shifted_suffix_keys(model: Any, key: torch.Tensor, shift: int) -> torch.Tensor:
    """Delta-RoPE of retained suffix keys ``[1, Hkv, S, D]`` (cache.py:47-77).

    Zero shift or an empty suffix returns a copy (cache.py:51-52).
    """
    require_cuda_tensors([key], "shifted_suffix_keys")
    _check_kv_layout([key], "shifted_suffix_keys")
    out = torch.empty(key.shape, dtype=key.dtype, device=key.device)
    if not key.shape[2] or not shift:
        out.copy_(key)
        return out
    table = _shift_table(model, key, shift)
    _, heads, rows, dim = key.shape
    hs, rs = kv_strides(key)
    lib = _lib.load()
    _lib.check(lib.kvr_rope_shift_layers(_lib.ptr_array([key]), _lib.ptr_array([out]), 1, heads, rows, dim,
                                         hs, rs, rows * dim, dim, table.data_ptr(),
                                         _lib.dtype_code(key.dtype), _lib.stream_handle(key.device)),
               "rope_shift_layers")
    return out


def shift_layers(model: Any, pairs, alignment: dict, recompute_end: int, old_tail_start: int):
    """New per-layer tensors of the edited length: prefix copied, retained tail
    moved up and its K re-rotated by ``position_shift``; rows
    ``[prefix, recompute_end)`` are left for the caller to recompute."""
    tensors = [t for pair in pairs for t in pair]
    device = require_cuda_tensors(tensors, "build_halo_cache")
    _check_kv_layout(tensors, "build_halo_cache")
    key = tensors[0]
    _, heads, old_rows, dim = key.shape
    new_rows = recompute_end + (old_rows - old_tail_start)
    if len(pairs) > _lib.MAX_LAYER_TENSORS // 2:
        raise ValueError("build_halo_cache: more layers than one launch takes")
    hs, rs = _uniform_strides(tensors, "build_halo_cache")
    shift = int(alignment["position_shift"])
    fresh = allocate_layers(len(pairs), heads, new_rows, dim, key.dtype, device)
    k_new = [k for k, _ in fresh]
    v_new = [v for _, v in fresh]
    if new_rows:
        table = _shift_table(model, key, shift) if shift and old_rows > old_tail_start else None
        from .engine import kernel_timer

        timer = kernel_timer()
        token = timer.start("shift_cache_layers") if timer else None
        lib = _lib.load()
        _lib.check(lib.kvr_shift_cache_layers(
            _lib.ptr_array([k for k, _ in pairs]), _lib.ptr_array([v for _, v in pairs]),
            _lib.ptr_array(k_new), _lib.ptr_array(v_new), len(pairs), heads, dim, new_rows,
            alignment["prefix"], old_tail_start, recompute_end, hs, rs, new_rows * dim, dim,
            table.data_ptr() if table is not None else None, 1 if table is not None else 0,
            _lib.dtype_code(key.dtype), _lib.stream_handle(device)), "shift_cache_layers")
        if token:
            timer.stop(token)
    return list(zip(k_new, v_new))


@torch.no_grad()
def build_halo_cache(model: Any, old_cache: Any, old_input_ids: torch.Tensor, new_input_ids: torch.Tensor,
                     halo_tokens: int):
    """Preserve the common prefix, refresh changed tokens/halo, then shift the
    tail (cache.py:103-144). Returns ``(cache, alignment metadata)``.

    One kernel writes every layer of the shifted cache. The changed boundary
    tokens and the halo (rows ``[prefix, new_suffix_start + halo)``) are then
    recomputed by the packed engine over that cache: each of those rows sees
    the prefix and the recomputed rows before it, and nothing after it, which
    is the reference's ``run_tokens_from_prefix`` over the prefix cache.
    """
    alignment = token_alignment(old_input_ids[0].cpu().numpy(), new_input_ids[0].cpu().numpy())
    halo = min(max(int(halo_tokens), 0), alignment["suffix"])
    recompute_end = alignment["new_suffix_start"] + halo
    old_tail_start = alignment["old_suffix_start"] + halo
    pairs = cache_layers(old_cache)
    layers = shift_layers(model, pairs, alignment, recompute_end, old_tail_start)
    if recompute_end > alignment["prefix"]:
        from .packed import refresh_owned_layers

        intervals = [(alignment["prefix"], recompute_end)]
        refresh_owned_layers(model, layers, new_input_ids, intervals)
    return make_cache(layers), {
        **alignment,
        "halo_tokens": halo,
        "recomputed_tokens": alignment["mandatory_changed_tokens"] + halo,
    }


def merge_intervals(intervals):
    """Sorted union of half-open intervals (cache.py:195-204)."""
    output = []
    for start, end in sorted((int(s), int(e)) for s, e in intervals if int(e) > int(s)):
        if output and start <= output[-1][1]:
            output[-1] = (output[-1][0], max(output[-1][1], end))
        else:
            output.append((start, end))
    return output
