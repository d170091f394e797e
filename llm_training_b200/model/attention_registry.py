"""Attention plugin registry: the drop-in boundary of the reference trainer.

Public API (what a trainer written against the reference's
model/attention_registry.py calls, :39-151): ``BaseAttention``,
``register_attention(*names)``, ``get_attention(name)``,
``build_attention(config)`` and ``available_attentions()``, with the same
contract - names compare case-insensitively with '-' and '_' equivalent, a
name already taken by another class raises ValueError, a class that is not a
BaseAttention raises TypeError, an unknown name raises KeyError listing the
known ones, a 'package.module:ClassName' string loads a class directly, and
``build_attention`` reads ``config.attention`` (default "vanilla").

Design.  One ``AttentionRegistry`` object holds the name table and the
plugin discovery state.  Discovery runs once, on the first lookup: every
module of this package (and any module named in ``extra_plugins``) is
imported so its ``@register_attention`` decorators run.  A plugin module that
fails to import is recorded in the ``DiscoveryReport`` (``discovery_errors()``)
instead of aborting the lookup - unlike the reference, where one broken module
(model/flash_attention.py:5) makes the first lookup of every name raise.
"""

from __future__ import annotations

import dataclasses
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


@dataclasses.dataclass
class DiscoveryReport:
    """Outcome of the plugin scan: modules imported and modules that failed."""

    imported: list = dataclasses.field(default_factory=list)
    failed: dict = dataclasses.field(default_factory=dict)  # module -> "Error: message"


class AttentionRegistry:
    """Canonical name -> attention class, filled by plugin modules on import."""

    def __init__(self, package: str, extra_plugins=()):
        self.package = package
        self.extra_plugins = list(extra_plugins)
        self._classes: dict[str, type] = {}
        self._report: DiscoveryReport | None = None

    @staticmethod
    def canonical(name: str) -> str:
        """'Sqrt-Block ' and 'sqrt_block' name the same attention."""
        return "_".join(name.strip().lower().split("-"))

    # -- registration ------------------------------------------------------------
    def add(self, cls, names) -> None:
        if not isinstance(cls, type) or not issubclass(cls, BaseAttention):
            raise TypeError(f"cannot register {cls!r}: attention plugins must derive from "
                            "BaseAttention (profilers find the attention layers through it)")
        keys = [self.canonical(n) for n in names]
        for key, name in zip(keys, names):
            holder = self._classes.get(key)
            if holder not in (None, cls):
                raise ValueError(f"attention name {name!r} is already registered to "
                                 f"{holder.__module__}.{holder.__qualname__}")
        self._classes.update(dict.fromkeys(keys, cls))

    def remove(self, name: str) -> None:
        self._classes.pop(self.canonical(name), None)

    # -- discovery ---------------------------------------------------------------
    def _plugin_modules(self):
        pkg = importlib.import_module(self.package)
        own = f"{self.package}.attention_registry"
        found = [f"{self.package}.{m.name}" for m in pkgutil.iter_modules(pkg.__path__)
                 if not m.name.startswith("_")]
        return [m for m in found if m != own] + self.extra_plugins

    def scan(self, force: bool = False) -> DiscoveryReport:
        """Import the plugin modules (once, or again with force=True)."""
        if self._report is not None and not force:
            return self._report
        report = DiscoveryReport()
        self._report = report  # plugins imported below look names up through us
        for module in self._plugin_modules():
            try:
                importlib.import_module(module)
            except Exception as exc:  # recorded: one broken plugin hides no other
                report.failed[module] = f"{type(exc).__name__}: {exc}"
            else:
                report.imported.append(module)
        return report

    # -- lookup ------------------------------------------------------------------
    def names(self) -> list:
        self.scan()
        return sorted(self._classes)

    def resolve(self, name: str) -> type:
        if ":" in name:
            return _class_from_spec(name)
        self.scan()
        cls = self._classes.get(self.canonical(name))
        if cls is None:
            raise KeyError(f"no attention is registered as {name!r} (known: "
                           f"{', '.join(self.names()) or 'none'}); a module in "
                           f"{self.package} that registers a BaseAttention subclass with "
                           "@register_attention(...) adds one")
        return cls


def _class_from_spec(spec: str) -> type:
    """'package.module:ClassName' -> the class, which must be a BaseAttention."""
    module_name, class_name = spec.split(":", 1)
    cls = getattr(importlib.import_module(module_name), class_name, None)
    if cls is None:
        raise ValueError(f"{module_name} defines no {class_name!r} (from attention spec "
                         f"{spec!r})")
    if not isinstance(cls, type) or not issubclass(cls, BaseAttention):
        raise TypeError(f"attention spec {spec!r} does not name a BaseAttention subclass")
    return cls


REGISTRY = AttentionRegistry(__name__.rsplit(".", 1)[0])


def register_attention(*names):
    """Class decorator: register the class under every name given."""

    def decorator(cls):
        REGISTRY.add(cls, names)
        return cls

    return decorator


def available_attentions():
    """Sorted canonical names of every registered attention."""
    return REGISTRY.names()


def get_attention(name):
    """The attention class registered as ``name``, or loaded from 'module:Class'."""
    return REGISTRY.resolve(name)


def build_attention(config, name=None):
    """An instance of the attention ``config.attention`` (or ``name``) names."""
    return get_attention(name if name is not None else getattr(config, "attention", "vanilla"))(
        config)


def discovery_errors():
    """Plugin modules that failed to import during discovery, with their error."""
    return dict(REGISTRY.scan().failed)
