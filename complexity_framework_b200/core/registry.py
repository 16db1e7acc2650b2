"""Name -> class registries for attention, MLP, normalisation and position modules.

Same registry names and decorator API as complexity/core/registry.py:22-129.
"""
from __future__ import annotations

from typing import Callable, Dict, Type


class Registry:
    def __init__(self, kind: str):
        self.kind = kind
        self._items: Dict[str, Type] = {}

    def register(self, name: str) -> Callable[[Type], Type]:
        def deco(cls: Type) -> Type:
            self._items[name.lower()] = cls
            return cls

        return deco

    def get(self, name: str) -> Type:
        key = str(name).lower()
        if key not in self._items:
            raise KeyError(f"unknown {self.kind} {name!r}; available: {sorted(self._items)}")
        return self._items[key]

    def build(self, name: str, *args, **kwargs):
        return self.get(name)(*args, **kwargs)

    def names(self):
        return sorted(self._items)

    def __contains__(self, name: str) -> bool:
        return str(name).lower() in self._items


ATTENTION_REGISTRY = Registry("attention")
MLP_REGISTRY = Registry("mlp")
NORMALIZATION_REGISTRY = Registry("normalization")
POSITION_REGISTRY = Registry("position")
MODEL_REGISTRY = Registry("model")

register_attention = ATTENTION_REGISTRY.register
register_mlp = MLP_REGISTRY.register
register_normalization = NORMALIZATION_REGISTRY.register
register_position = POSITION_REGISTRY.register
register_model = MODEL_REGISTRY.register
