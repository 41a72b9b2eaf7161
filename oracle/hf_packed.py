"""The reference's packed executor restated on the transformers modules.

TEST AND BASELINE INFRASTRUCTURE ONLY (the product never imports it). It runs
the same library calls as the reference's default path
(kernels/packed_cache.py:225-298): an owned copy of every cache layer made the
way ``clone_cache`` makes it (cache.py:31-44: ``.clone()`` then
``DynamicCache.update``, whose ``torch.cat`` copies again), a shallow model
view whose attention implementation is a registered function (packed_cache.py:
85-120), cache layers that ``index_copy_`` the fresh K/V rows before returning
the full tensors (packed_cache.py:166-200), and SDPA with the dense
``[1, 1, B, N]`` absolute-causal mask (packed_cache.py:47-67, 203-207), which
makes transformers' ``sdpa_attention_forward`` materialise ``repeat_kv``.

It serves as (1) the timed CPU reference arm of ``bench.py`` and (2) the GPU
comparator ("the reference CUDA SDPA path") on the box, where the reference
package itself is not installed.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass
from threading import Lock

import torch

_NAME = "oracle_packed_absolute_attention"
_LOCK = Lock()


@dataclass
class _Context:
    positions: torch.Tensor
    length: int
    mask: torch.Tensor


def _attention(module, query, key, value, attention_mask, *, scaling=None, dropout=0.0,
               oracle_packed_context=None, **kwargs):
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    ctx = oracle_packed_context
    return sdpa_attention_forward(module, query, key, value, ctx.mask, dropout=0.0, scaling=scaling,
                                  is_causal=False)


def _register():
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    with _LOCK:
        if _NAME not in ALL_ATTENTION_FUNCTIONS:
            ALL_ATTENTION_FUNCTIONS.register(_NAME, _attention)


def _layer_class():
    from transformers.cache_utils import DynamicLayer

    class PackedLayer(DynamicLayer):
        def __init__(self, key, value, ctx):
            super().__init__()
            self.keys, self.values = key, value
            self.dtype, self.device = key.dtype, key.device
            self.is_initialized = True
            self.ctx = ctx

        def get_mask_sizes(self, *args, **kwargs):
            return self.ctx.length, 0

        def update(self, key_states, value_states, *args, **kwargs):
            self.keys.index_copy_(2, self.ctx.positions, key_states)
            self.values.index_copy_(2, self.ctx.positions, value_states)
            return self.keys, self.values

    return PackedLayer


def _view(base):
    _register()
    config = copy.deepcopy(base.config)
    config._attn_implementation = _NAME
    view = copy.copy(base)
    view._modules = base._modules.copy()
    view.config = config
    layers = []
    for original in base.layers:
        layer = copy.copy(original)
        layer._modules = original._modules.copy()
        if hasattr(layer, "config"):
            layer.config = config
        attention = copy.copy(original.self_attn)
        attention._modules = original.self_attn._modules.copy()
        attention.config = config
        layer._modules["self_attn"] = attention
        layers.append(layer)
    view._modules["layers"] = torch.nn.ModuleList(layers)
    return view


def clone_layers_like_reference(layers):
    """``clone_cache`` on this transformers: clone, then ``DynamicCache.update``
    (``torch.cat`` onto an empty tensor), i.e. two copies per tensor."""
    from transformers.cache_utils import DynamicCache

    cache = DynamicCache()
    for index, (key, value) in enumerate(layers):
        cache.update(key.clone(), value.clone(), index)
    return [(layer.keys, layer.values) for layer in cache.layers]


@torch.no_grad()
def packed_refresh_hf(base, base_layers, ids, positions):
    """Refresh ``positions`` through every layer of ``base`` (a LlamaModel or
    Qwen3Model); returns new ``(K, V)`` layers. ``ids``: ``[1, N]`` or ``[N]``."""
    from transformers.cache_utils import Cache

    device = base_layers[0][0].device
    ids = torch.as_tensor(ids, device=device).reshape(1, -1)
    length = ids.shape[1]
    pos = torch.tensor([int(p) for p in positions], dtype=torch.long, device=device)
    mask = (torch.arange(length, device=device)[None, :] <= pos[:, None])[None, None]
    ctx = _Context(pos, length, mask)
    owned = clone_layers_like_reference(base_layers)
    layer_cls = _layer_class()
    cache = Cache(layers=[layer_cls(k, v, ctx) for k, v in owned])
    view = _view(base)
    view(input_ids=ids.index_select(1, pos), position_ids=pos.unsqueeze(0), cache_position=pos,
         past_key_values=cache, use_cache=True, return_dict=True, oracle_packed_context=ctx)
    return owned
