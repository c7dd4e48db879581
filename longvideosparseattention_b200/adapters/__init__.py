"""Adapter registry (mirror of lvsa/adapters/__init__.py:15-62)."""

from importlib import import_module
from typing import Dict, Tuple, Type

from .base import ModelAdapter

_ADAPTER_REGISTRY: Dict[str, Tuple[str, str]] = {
    "wan": ("longvideosparseattention_b200.adapters.wan", "WanAdapter"),
    "hunyuan_video": ("longvideosparseattention_b200.adapters.hunyuan_video", "HunyuanVideoAdapter"),
    "cogvideox": ("longvideosparseattention_b200.adapters.cogvideox", "CogVideoXAdapter"),
}


def get_adapter(name: str) -> ModelAdapter:
    """Instantiate a registered adapter; KeyError names the available ones."""
    if name not in _ADAPTER_REGISTRY:
        raise KeyError(f"Unknown adapter {name!r}. Available adapters: {', '.join(sorted(_ADAPTER_REGISTRY))}")
    module_path, class_name = _ADAPTER_REGISTRY[name]
    cls: Type[ModelAdapter] = getattr(import_module(module_path), class_name)
    return cls()


def register_adapter(name: str, module_path: str, class_name: str) -> None:
    """Register (or replace) an adapter by import path."""
    _ADAPTER_REGISTRY[name] = (module_path, class_name)


__all__ = ["ModelAdapter", "get_adapter", "register_adapter"]
