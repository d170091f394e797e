"""Attention plugin registry: the drop-in boundary of the reference trainer.

Same public API and semantics as the reference's model/attention_registry.py:
``BaseAttention`` (:39-56), ``register_attention`` (:67-90; names normalised
case-insensitively with '-' == '_', :63-64; a name already bound to another
class raises ValueError, :80-86; non-BaseAttention classes raise TypeError,
:74-78), lazy package discovery (:93-107), the ``module:Class`` escape hatch
(:110-120), ``available_attentions`` (:123-126), ``get_attention`` (:129-141,
KeyError listing the registered names) and ``build_attention`` (:144-151,
``config.attention`` defaulting to "vanilla").

One deliberate difference: discovery imports each module inside a try block
and records (rather than propagates) an import failure.  In the reference a
single broken module (model/flash_attention.py:5) makes the first lookup raise
for every attention.  ``discovery_errors()`` reports what was skipped.
"""

from __future__ import annotations

import importlib
import pkgutil

import torch.nn as nn


class BaseAttention(nn.Module):
    """Base class of every attention implementation.

    Profilers hook every instance of this class (forward pre/post and full
    backward pre/post hooks), so subclasses must take and return plain
    tensors: ``forward(X: (B, T, C)) -> (B, T, C)``.
    """

    def __init__(self, config):
        super().__init__()
        self.config = config

    def forward(self, X):
        raise NotImplementedError


_REGISTRY: dict[str, type] = {}
_discovered = False
_discovery_errors: dict[str, str] = {}


def _normalize(name):
    return name.strip().lower().replace("-", "_")


def register_attention(*names):
    """Class decorator registering an attention under one or more names."""

    def decorator(cls):
        if not (isinstance(cls, type) and issubclass(cls, BaseAttention)):
            raise TypeError(
                f"{getattr(cls, '__name__', cls)} must subclass BaseAttention to be registered "
                "(profilers find attention layers by that base class)")
        for name in names:
            key = _normalize(name)
            existing = _REGISTRY.get(key)
            if existing is not None and existing is not cls:
                raise ValueError(
                    f"attention name {name!r} is already registered to "
                    f"{existing.__module__}.{existing.__name__}")
            _REGISTRY[key] = cls
        return cls

    return decorator


def _discover():
    """Import every module of this package once so that decorators run."""
    global _discovered
    if _discovered:
        return
    _discovered = True  # set first: the imports below re-enter this module
    package = importlib.import_module(__package__)
    for info in pkgutil.walk_packages(package.__path__, prefix=f"{__package__}."):
        if info.name == __name__ or info.name.rsplit(".", 1)[-1].startswith("_"):
            continue
        try:
            importlib.import_module(info.name)
        except Exception as exc:  # a broken plugin must not hide the others
            _discovery_errors[info.name] = f"{type(exc).__name__}: {exc}"


def discovery_errors():
    """Modules skipped by discovery, with the error each raised."""
    _discover()
    return dict(_discovery_errors)


def _load_from_path(spec):
    """Resolve a 'module.path:ClassName' spec into a class."""
    module_path, _, class_name = spec.partition(":")
    module = importlib.import_module(module_path)
    try:
        cls = getattr(module, class_name)
    except AttributeError:
        raise ValueError(f"module {module_path!r} has no attribute {class_name!r}") from None
    if not (isinstance(cls, type) and issubclass(cls, BaseAttention)):
        raise TypeError(f"{spec} must be a BaseAttention subclass")
    return cls


def available_attentions():
    """Sorted list of registered names."""
    _discover()
    return sorted(_REGISTRY)


def get_attention(name):
    """Look up a registered attention class by name (or 'module:Class' path)."""
    if ":" in name:
        return _load_from_path(name)
    _discover()
    try:
        return _REGISTRY[_normalize(name)]
    except KeyError:
        raise KeyError(
            f"unknown attention {name!r}; available: {', '.join(available_attentions())}. "
            "Add a new one by dropping a module in this package with a "
            "@register_attention(...) BaseAttention subclass.") from None


def build_attention(config, name=None):
    """Instantiate the attention selected by ``config.attention`` (or ``name``)."""
    if name is None:
        name = getattr(config, "attention", "vanilla")
    return get_attention(name)(config)
