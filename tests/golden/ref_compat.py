"""Run the upstream reference (yh0903/budgeted-kv-cache-repair) on transformers 5.5.

Fixture-generation helper only. It imports the reference package from a source
tree given at run time and patches four version-dependent surfaces; no
arithmetic of the reference or of transformers is changed:

1. ``Cache``/``DynamicCache`` ``__getitem__`` and ``__iter__`` return
   ``(keys, values)`` pairs, the 4.57 tuple protocol the reference indexes and
   unpacks with (``cache.py:37``, ``kernels/packed_cache.py:150``).
2. The reference's hard version pin (``kernels/packed_cache.py:124-125``,
   ``api.py:139-140``) sees ``"4.57.6"``.
3. ``config.rope_scaling`` aliases ``rope_parameters`` in 5.5 and is never
   ``None``; the reference's default-RoPE check (``kernels/packed_cache.py:139``,
   ``api.py:148``) sees ``None`` while ``rope_type`` is ``"default"``.
4. transformers 5.5 calls ``layer.update(k, v)`` without ``cache_kwargs``;
   ``_PackedLayer.update`` (``kernels/packed_cache.py:179-188``) receives the
   request's own positions tensor as ``cache_position``, which is what 4.57 passed.
"""

from __future__ import annotations

import sys
import types


def load_reference(src_root: str):
    """Import ``kv_cache_repair`` from ``src_root`` with the four patches applied."""
    if src_root not in sys.path:
        sys.path.insert(0, src_root)
    from transformers.cache_utils import Cache, DynamicCache

    def _getitem(self, index):
        layer = self.layers[index]
        return layer.keys, layer.values

    def _iter(self):
        for layer in self.layers:
            yield layer.keys, layer.values

    for cls in (Cache, DynamicCache):
        cls.__getitem__ = _getitem
        cls.__iter__ = _iter

    from transformers import LlamaForCausalLM  # noqa: F401  (settles the lazy module)
    import kv_cache_repair.api as api
    import kv_cache_repair.kernels.packed_cache as packed

    pinned = types.SimpleNamespace(__version__="4.57.6")
    packed.transformers = pinned
    original_check_model = api._check_model
    original_qualify = packed._qualify

    class _DefaultRopeView:
        """Config proxy reporting ``rope_scaling=None`` for default RoPE only."""

        def __init__(self, config):
            object.__setattr__(self, "_config", config)

        def __getattr__(self, name):
            value = getattr(self._config, name)
            if name == "rope_scaling" and isinstance(value, dict) and value.get("rope_type") == "default":
                return None
            return value

    def _with_default_rope(model, call):
        config = model.config
        model.__dict__["config"] = _DefaultRopeView(config)
        try:
            return call()
        finally:
            model.__dict__["config"] = config

    def check_model(model):
        # transformers replaces its lazy module object in sys.modules on first
        # attribute import, so patch whichever object is current at call time.
        live = sys.modules["transformers"]
        saved = live.__version__
        live.__version__ = "4.57.6"
        try:
            return _with_default_rope(model, lambda: original_check_model(model))
        finally:
            live.__version__ = saved

    def qualify(shim, edited_ids, base_cache, attention_backend, writeback_backend):
        return _with_default_rope(
            shim.generator,
            lambda: original_qualify(shim, edited_ids, base_cache, attention_backend, writeback_backend),
        )

    api._check_model = check_model
    packed._qualify = qualify

    original_update = packed._PackedLayer.update
    if not getattr(original_update, "_ref_compat", False):
        def update(self, key_states, value_states, cache_kwargs=None, *args, **kwargs):
            if not isinstance(cache_kwargs, dict):
                cache_kwargs = {"cache_position": self._context.positions}
            return original_update(self, key_states, value_states, cache_kwargs)

        update._ref_compat = True
        packed._PackedLayer.update = update
    import kv_cache_repair
    return kv_cache_repair
