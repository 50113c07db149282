"""Llama-style dense decoder adapter (Llama-3, Mistral, Qwen2/Qwen3 dense).

The reference ships TP adapters only for the Qwen hybrid and LFM2 families
(voodoo_quant/arch/qwen.py, lfm2.py) and refuses every other model under TP
(parallel.py:685-694), which rules out the dense-decoder benchmark shapes.
Policy: q/k/v column-parallel by whole heads, o_proj row-parallel; gate/up
column-parallel, down_proj row-parallel (256-aligned, possibly uneven);
embedding and lm_head vocabulary-parallel (handled by tp_patch_model).
"""

from __future__ import annotations

import torch.nn as nn

from voodoo_quant.arch import register
from voodoo_quant.arch.base import ArchAdapter


@register
class LlamaDenseAdapter(ArchAdapter):
    hf_model_types = ("llama", "mistral", "qwen2", "qwen3")
    ggml_archs = ("llama", "qwen2", "qwen3")
    attention_segments = frozenset({"self_attn"})

    @classmethod
    def shard_layer(cls, layer) -> list[str]:
        from voodoo_quant.parallel import tp_attention_dense, tp_mlp

        handled = []
        attn = getattr(layer, "self_attn", None)
        if isinstance(attn, nn.Module):
            cfg = getattr(attn, "config", None)
            nh = getattr(cfg, "num_attention_heads", None) or getattr(attn, "num_heads")
            nkv = getattr(cfg, "num_key_value_heads", None) or getattr(attn, "num_key_value_heads", nh)
            hd = getattr(attn, "head_dim", None) or attn.q_proj.out_features // nh
            tp_attention_dense(attn, nh, nkv, hd)
            handled.append("self_attn")
        if getattr(layer, "mlp", None) is not None:
            tp_mlp(layer.mlp)
            handled.append("mlp")
        return handled
