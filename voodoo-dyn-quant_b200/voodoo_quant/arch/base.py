"""Architecture adapter base class (same contract as the reference's
voodoo_quant/arch/base.py:32-83): an adapter owns the tensor-parallel sharding
policy of one model family, expressed with the primitives of
:mod:`voodoo_quant.parallel`."""

from __future__ import annotations

from typing import Optional

DEFAULT_ATTENTION_SEGMENTS: frozenset[str] = frozenset({"self_attn", "linear_attn", "attn", "conv", "shortconv"})


class ArchAdapter:
    hf_model_types: tuple[str, ...] = ()
    ggml_archs: tuple[str, ...] = ()
    attention_segments: frozenset[str] = DEFAULT_ATTENTION_SEGMENTS

    @classmethod
    def matches_config(cls, config) -> bool:
        return getattr(config, "model_type", None) in cls.hf_model_types

    @classmethod
    def matches_gguf_arch(cls, arch: str) -> bool:
        return arch in cls.ggml_archs

    @classmethod
    def shard_layer(cls, layer) -> list[str]:
        return []

    @classmethod
    def gguf_name(cls, hf_name: str) -> Optional[str]:
        return None

    @classmethod
    def transpose_embedding(cls) -> bool:
        return False

    @classmethod
    def is_attention_tensor(cls, hf_name: str) -> bool:
        return any(seg in cls.attention_segments for seg in hf_name.split("."))
