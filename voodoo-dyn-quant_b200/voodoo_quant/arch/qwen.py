"""Qwen3.5-family hybrid adapter: Gated DeltaNet (linear attention) layers
and gated full-attention layers (the reference's QwenHybridAdapter,
voodoo_quant/arch/qwen.py).

Policy, through the primitives of :mod:`voodoo_quant.parallel`:
``linear_attn`` by value heads (``tp_ssm``), ``self_attn`` by whole heads
with each head's q and gate together (``tp_attention``), MLP gate/up
column-parallel and down row-parallel (``tp_mlp``); embedding and lm_head
vocabulary-parallel (``tp_patch_model``).  GGUF names are left to the
exporter's own table (``gguf_name`` returns None, as in the reference).
"""

from __future__ import annotations

import torch.nn as nn

from voodoo_quant.arch import register
from voodoo_quant.arch.base import ArchAdapter


@register
class QwenHybridAdapter(ArchAdapter):
    hf_model_types = ("qwen3_5", "qwen3_5_text", "qwen3_6", "qwen3_8")
    ggml_archs = ("qwen35", "qwen36", "qwen38")
    attention_segments = frozenset({"self_attn", "linear_attn"})

    @classmethod
    def shard_layer(cls, layer) -> list[str]:
        from voodoo_quant.parallel import tp_attention, tp_mlp, tp_ssm

        handled = []
        if isinstance(getattr(layer, "linear_attn", None), nn.Module):
            tp_ssm(layer.linear_attn)
            handled.append("linear_attn")
        if isinstance(getattr(layer, "self_attn", None), nn.Module):
            tp_attention(layer.self_attn)
            handled.append("self_attn")
        if getattr(layer, "mlp", None) is not None:
            tp_mlp(layer.mlp)
            handled.append("mlp")
        return handled
