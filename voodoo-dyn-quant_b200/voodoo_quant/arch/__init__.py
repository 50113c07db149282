"""Architecture adapter registry (the reference's plugin mechanism,
voodoo_quant/arch/__init__.py:33-72): adapters register with ``@register``
and are found by the model config's ``model_type``."""

from __future__ import annotations

from typing import Optional, Type

from voodoo_quant.arch.base import ArchAdapter, DEFAULT_ATTENTION_SEGMENTS  # noqa: F401


class NullAdapter(ArchAdapter):
    @classmethod
    def shard_layer(cls, layer) -> list[str]:
        return []


_ADAPTERS: list[Type[ArchAdapter]] = []
_REGISTERED_NAMES: set[str] = set()


def register(adapter_cls: Type[ArchAdapter]) -> Type[ArchAdapter]:
    if adapter_cls.__name__ not in _REGISTERED_NAMES:
        _ADAPTERS.append(adapter_cls)
        _REGISTERED_NAMES.add(adapter_cls.__name__)
    return adapter_cls


def _autoload() -> None:
    import importlib
    import pkgutil

    for mod in pkgutil.iter_modules(__path__):
        if mod.name not in ("base", "__init__"):
            importlib.import_module(f"{__name__}.{mod.name}")


def adapters() -> list[Type[ArchAdapter]]:
    if not _ADAPTERS:
        _autoload()
    return list(_ADAPTERS)


def adapter_for_config(config) -> Optional[Type[ArchAdapter]]:
    cfg = getattr(config, "text_config", config)
    for a in adapters():
        if a.matches_config(cfg):
            return a
    return None


def adapter_for_model(model) -> Optional[Type[ArchAdapter]]:
    cfg = getattr(model, "config", None)
    return None if cfg is None else adapter_for_config(cfg)


def adapter_for_gguf_arch(arch: str) -> Optional[Type[ArchAdapter]]:
    for a in adapters():
        if a.matches_gguf_arch(arch):
            return a
    return None
