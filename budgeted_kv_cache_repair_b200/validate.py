"""Contract checks shared by the packed executor and the cache operators.

Each check raises ``ValueError`` before any device work, with the reference's
rules (kernels/executor.py:19-70, kernels/packed_cache.py:123-163,
api.py:135-166, kernels/writeback.py:6-15).
"""

from __future__ import annotations

import weakref
from itertools import repeat
from numbers import Integral
from operator import attrgetter, is_not
from typing import Any, Sequence

import torch

from . import registry


def cache_layers(cache: Any) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """``(K, V)`` of every layer of a transformers Cache (4.57 or 5.x) or a
    sequence of pairs, without copying."""
    layers = getattr(cache, "layers", None)
    if layers is not None and all(hasattr(layer, "keys") and hasattr(layer, "values") for layer in layers):
        return [(layer.keys, layer.values) for layer in layers]
    try:
        count = len(cache)
    except TypeError as exc:
        raise ValueError("base_cache must expose indexed K/V layers") from exc
    out = []
    for index in range(count):
        try:
            key, value = cache[index][:2]
        except (TypeError, ValueError, IndexError) as exc:
            raise ValueError(f"cache layer {index} must contain one K/V pair") from exc
        out.append((key, value))
    return out


# Per-layer rules of the reference's cache check (kernels/executor.py:19-47),
# in the order it applies them; the first rule a layer breaks names the fault.
# The messages are the contract, the table is this module's own.
_LAYER_RULES = (
    (lambda k, v, n: isinstance(k, torch.Tensor) and isinstance(v, torch.Tensor),
     "cache layer {i} K/V must be tensors"),
    (lambda k, v, n: k.ndim == 4 and v.ndim == 4,
     "cache layer {i} K/V must have rank four"),
    (lambda k, v, n: k.shape == v.shape and k.dtype == v.dtype and k.device == v.device,
     "cache layer {i} K/V geometry, dtype, and device must agree"),
    (lambda k, v, n: k.shape[0] == 1 and k.shape[2] == n,
     "cache layer {i} must match the single-batch edited token length"),
    (lambda k, v, n: k.shape[1] > 0 and k.shape[3] > 0 and k.is_floating_point(),
     "cache layer {i} requires nonempty floating-point KV heads"),
)


def validate_cache(cache: Any, logical_length: int) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Rank-4 ``[1, Hkv, N, D]`` floating K/V, one geometry and dtype on every
    layer. Returns the layer pairs.

    Every layer is run through the rule table; its (shape, dtype) signature
    must then equal the first layer's.
    """
    layers = cache_layers(cache)
    if not layers:
        raise ValueError("base_cache must contain at least one K/V layer")
    # Fast path: every K and V a tensor of one (shape, dtype, device) that
    # passes the rules; otherwise the rule table below names the fault.
    try:
        kinds = {(type(t), t.shape, t.dtype, t.device) for pair in layers for t in pair}
    except AttributeError:
        kinds = ()
    if len(kinds) == 1:
        key, value = layers[0]
        if isinstance(key, torch.Tensor) and all(rule(key, value, logical_length) for rule, _ in _LAYER_RULES):
            return layers
    signatures = set()
    for index, (key, value) in enumerate(layers):
        broken = next((text for rule, text in _LAYER_RULES if not rule(key, value, logical_length)), None)
        if broken is not None:
            raise ValueError(broken.format(i=index))
        signatures.add((tuple(key.shape), key.dtype))
        if len(signatures) > 1:
            raise ValueError("cache layers must have regular shapes and matching dtypes")
    return layers


def validate_intervals(intervals: Sequence[tuple[int, int]], logical_length: int) -> tuple[tuple[int, int], ...]:
    """Sorted, disjoint, maximal (non-adjacent) half-open ranges (kernels/executor.py:50-70)."""
    if not isinstance(intervals, (list, tuple)):
        raise ValueError("intervals must be a list or tuple of maximal half-open ranges")
    result = []
    previous_end = -1
    for interval in intervals:
        if not isinstance(interval, (tuple, list)) or len(interval) != 2:
            raise ValueError("each interval must contain exactly a start and end")
        start, end = interval
        if type(start) is not int or type(end) is not int:  # plain ints skip the ABC checks
            if any(isinstance(v, bool) or not isinstance(v, Integral) for v in interval):
                raise ValueError("interval bounds must be integers, not booleans")
            start, end = int(start), int(end)
        if not 0 <= start < end <= logical_length:
            raise ValueError("interval bounds must satisfy 0 <= start < end <= token length")
        if start <= previous_end:
            raise ValueError("intervals must be sorted, disjoint, and maximal (no adjacent ranges)")
        result.append((start, end))
        previous_end = end
    return tuple(result)


def nonoverlapping_layout(tensor: torch.Tensor) -> bool:
    """Sufficient proof that no two elements share storage (kernels/writeback.py:6-15)."""
    extent = 1
    for stride, size in sorted(zip(tensor.stride(), tensor.shape)):
        if size > 1:
            if stride < extent:
                return False
            extent += (size - 1) * stride
    return True


def kv_strides(tensor: torch.Tensor) -> tuple[int, int]:
    """(head_stride, row_stride) of a ``[1, H, N, D]`` tensor with unit D stride."""
    if tensor.stride(3) != 1 and tensor.shape[3] > 1:
        raise ValueError("cache tensors need a unit stride along head_dim")
    return tensor.stride(1), tensor.stride(2)


def require_cuda_tensors(tensors, what: str) -> torch.device:
    device = None
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError(f"{what} requires CUDA tensors (the B200 engine has no CPU path)")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError(f"{what}: all tensors must share one CUDA device")
    return device


class _ModuleScan:
    """Flattened module/parameter lists of one model, so per-call checks need
    no recursive traversal; rebuilt when the decoder's structure changes."""

    __slots__ = ("epoch", "modules", "in_base", "params", "param_list", "states", "base_states",
                 "param_state")

    def __init__(self, model, base, epoch):
        self.epoch = epoch
        base_ids = {id(m) for m in base.modules()}
        self.modules = list(model.modules())
        registry.watch(self.modules)
        self.in_base = [id(m) in base_ids for m in self.modules]
        self.params = [(p, inb) for m, inb in zip(self.modules, self.in_base)
                       for p in m._parameters.values() if p is not None]
        self.param_list = [p for p, _ in self.params]
        # The modules' attribute dicts (the objects themselves, so a later
        # per-instance forward or hook shows up in them).
        self.states = [m.__dict__ for m in self.modules]
        self.base_states = [m.__dict__ for m, inb in zip(self.modules, self.in_base) if inb]
        self.param_state = None


_scans: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()


_training = attrgetter("training")


def _any_hook(states) -> bool:
    """Some module's attribute dict holds a non-None ``_hf_hook`` (an
    accelerate dispatch/offload hook); the scan runs at C level."""
    return any(map(is_not, map(dict.get, states, repeat("_hf_hook")), repeat(None)))


def _any_forward(states) -> bool:
    """Some module's attribute dict holds a per-instance ``forward``."""
    return any(map(dict.__contains__, states, repeat("forward")))


def _check_modules(model, base, device, dtype):
    # The module list, parameters and attribute dicts are re-collected once a
    # submodule or parameter of a watched model was registered or replaced
    # since the last scan (registry.epoch); the checks below run on every call.
    epoch = registry.epoch()
    scan = _scans.get(model)
    if scan is None or scan.epoch != epoch:
        scan = _ModuleScan(model, base, epoch)
        _scans[model] = scan
    if any(map(_training, scan.modules)):
        raise ValueError("packed executor requires eval mode on all decoder modules")
    if _any_hook(scan.states):
        raise ValueError("packed executor does not support dispatch/offload hooks")
    if _any_forward(scan.base_states):
        raise ValueError("packed executor does not support per-instance decoder forward overrides")
    # Parameter placement only needs re-checking when some parameter moved.
    state = (device, dtype, tuple(map(torch.Tensor.data_ptr, scan.param_list)))
    if scan.param_state != state:
        for p, in_base in scan.params:
            if p.device != device:
                raise ValueError("packed executor requires all model parameters on the request device")
            if in_base and p.dtype != dtype:
                raise ValueError("model parameters and cache must share one bfloat16/float16 dtype")
        scan.param_state = state


def qualify_model(model: Any, base: Any, layer_count: int, device: torch.device, dtype: torch.dtype) -> None:
    """Model contract of the packed path (kernels/packed_cache.py:123-163, api.py:135-166).

    Exact native dense Llama/Qwen3 classes, eval mode, default RoPE, full
    attention, every parameter on the request device, no offload hooks or
    per-instance forwards, and the arithmetic the kernels implement.
    """
    from transformers.models.llama.modeling_llama import LlamaForCausalLM, LlamaModel
    from transformers.models.qwen3.modeling_qwen3 import Qwen3ForCausalLM, Qwen3Model

    pairs = {(LlamaForCausalLM, LlamaModel), (Qwen3ForCausalLM, Qwen3Model)}
    if (type(model), type(base)) not in pairs and type(model) not in (LlamaModel, Qwen3Model):
        raise ValueError("packed executor requires exact native dense Llama or Qwen3 classes")
    config = model.config
    if config.num_hidden_layers != layer_count or len(base.layers) != layer_count:
        raise ValueError("model and cache layer counts must agree")
    check_model_arithmetic(config, base, "packed executor")
    _check_modules(model, base, device, dtype)
    if getattr(model, "is_quantized", False):
        raise ValueError("packed executor does not support quantized models")


def check_model_arithmetic(config: Any, base: Any, who: str) -> None:
    """The model features the kernels implement: default fixed RoPE, full
    attention on every layer, SiLU-gated MLP, bias-free projections
    (kernels/packed_cache.py:123-163, api.py:148-155). Raises ``ValueError``
    naming ``who``; reads only the config and module attributes (no device
    work), so the public API runs it before positional correction."""
    rope = getattr(config, "rope_parameters", None)
    rope_type = rope.get("rope_type", "default") if isinstance(rope, dict) else None
    if rope is None:
        scaling = getattr(config, "rope_scaling", None)
        rope_type = "default" if scaling is None else scaling.get("rope_type", scaling.get("type"))
    if rope_type != "default" or getattr(getattr(base, "rotary_emb", None), "rope_type", "default") != "default":
        raise ValueError(f"{who} supports default fixed RoPE only")
    if getattr(config, "use_sliding_window", False) or getattr(base, "has_sliding_layers", False):
        raise ValueError(f"{who} requires full attention, not sliding or hybrid attention")
    if any(kind != "full_attention" for kind in getattr(config, "layer_types", []) or []):
        raise ValueError(f"{who} requires full attention, not sliding or hybrid attention")
    if getattr(config, "hidden_act", "silu") != "silu":
        raise ValueError(f"{who} implements the SiLU-gated MLP only")
    if getattr(config, "attention_bias", False) or getattr(config, "mlp_bias", False):
        raise ValueError(f"{who} implements bias-free projections only")
