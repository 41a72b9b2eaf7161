"""Count of parameter, buffer and submodule registrations on watched modules.

torch calls its global registration hooks whenever any module gains or
replaces a parameter, buffer or child module (``Module.__setattr__``,
``register_parameter``, ``register_buffer``, ``add_module``). The engine's
cached model views and the per-call module scan watch the modules of the
models they were built from, remember the count they were built at, and are
rebuilt when it has moved: a parameter object swapped anywhere in such a
model since then (not only an in-place change, which data pointers and
version counters already show) can never be computed with from a stale cache.
Registrations on other modules (models being built, views another library
makes of a model) are not counted. The hooks only count; they never change
what is registered.
"""

from __future__ import annotations

import weakref

import torch.nn.modules.module as _module

_epoch = [0]
_watched: "weakref.WeakSet" = weakref.WeakSet()


def _count(module, *_args) -> None:
    try:
        watched = module in _watched
    except TypeError:  # a module class without a hash is never watched
        watched = False
    if watched:
        _epoch[0] += 1
    return None


_module.register_module_parameter_registration_hook(_count)
_module.register_module_buffer_registration_hook(_count)
_module.register_module_module_registration_hook(_count)


def watch(modules) -> None:
    """Count registrations on these modules from now on."""
    _watched.update(modules)


def epoch() -> int:
    """Registrations seen on watched modules so far."""
    return _epoch[0]
