"""LFM2 / LFM2.5 (LiquidAI) adapter: short-convolution and GQA attention
layers, SwiGLU MLP named ``feed_forward.w1/w3/w2`` (the reference's
LFM2Adapter, voodoo_quant/arch/lfm2.py).

Tensor parallelism: attention q/k/v column-parallel and ``out_proj``
row-parallel; the short convolution by hidden channels -- ``in_proj`` emits
[B | C | x] thirds of ``hidden`` channels each, the rank keeps its channel
slice of every third (same order, so the forward's ``chunk(3)`` still
splits it), the depthwise conv is rebuilt on those channels and ``out_proj``
is row-parallel; ``w1`` / ``w3`` column-parallel, ``w2`` row-parallel.
Every sharded block's input passes the exact-gradient operator.
GGUF names follow llama.cpp's ``lfm2`` tensor names (a format contract);
the token embedding is stored transposed there.
"""

from __future__ import annotations

import re
from typing import Optional

import torch
import torch.nn as nn

from voodoo_quant.arch import register
from voodoo_quant.arch.base import ArchAdapter

_GGUF_PATTERNS = [
    (re.compile(r"^model\.layers\.(\d+)\.conv\.(in_proj|out_proj)\.weight$"), "blk.{0}.shortconv.{1}.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.conv\.conv\.weight$"), "blk.{0}.shortconv.conv.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.self_attn\.q_proj\.weight$"), "blk.{0}.attn_q.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.self_attn\.k_proj\.weight$"), "blk.{0}.attn_k.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.self_attn\.v_proj\.weight$"), "blk.{0}.attn_v.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.self_attn\.out_proj\.weight$"), "blk.{0}.attn_output.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.self_attn\.q_layernorm\.weight$"), "blk.{0}.attn_q_norm.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.self_attn\.k_layernorm\.weight$"), "blk.{0}.attn_k_norm.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.feed_forward\.w1\.weight$"), "blk.{0}.ffn_gate.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.feed_forward\.w3\.weight$"), "blk.{0}.ffn_up.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.feed_forward\.w2\.weight$"), "blk.{0}.ffn_down.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.operator_norm\.weight$"), "blk.{0}.attn_norm.weight"),
    (re.compile(r"^model\.layers\.(\d+)\.ffn_norm\.weight$"), "blk.{0}.ffn_norm.weight"),
    (re.compile(r"^model\.embed_tokens\.weight$"), "token_embd.weight"),
    (re.compile(r"^model\.embedding_norm\.weight$"), "token_embd_norm.weight"),
]


def _split(n: int, tp: int, what: str) -> int:
    if n % tp:
        raise ValueError(f"{what} {n} not divisible by tp={tp}")
    return n // tp


@register
class LFM2Adapter(ArchAdapter):
    hf_model_types = ("lfm2",)
    ggml_archs = ("lfm2",)
    attention_segments = frozenset({"self_attn", "conv"})  # short-conv layers count as attention-side

    @classmethod
    def shard_layer(cls, layer) -> list[str]:
        from voodoo_quant.parallel import TP, _install_input_copy, _shard_child

        tp, r = TP.world_size, TP.rank
        if tp < 2:
            return []
        handled = []
        attn = getattr(layer, "self_attn", None)
        if isinstance(attn, nn.Module) and getattr(attn, "q_proj", None) is not None:
            for name in ("q_proj", "k_proj", "v_proj"):
                n = _split(getattr(attn, name).out_features, tp, name + " out")
                _shard_child(attn, name, row_offset=r * n, row_len=n)
            n = _split(attn.out_proj.in_features, tp, "out_proj in")
            _shard_child(attn, "out_proj", col_offset=r * n, col_len=n)
            _install_input_copy(attn)
            handled.append("self_attn")
        conv = getattr(layer, "conv", None)
        if isinstance(conv, nn.Module) and getattr(conv, "in_proj", None) is not None:
            hidden = conv.in_proj.in_features
            lh = _split(hidden, tp, "short-conv hidden")
            keep = torch.cat([torch.arange(j * hidden + r * lh, j * hidden + (r + 1) * lh) for j in range(3)])
            _shard_child(conv, "in_proj", row_index=keep)
            dw = conv.conv
            if isinstance(dw, nn.Conv1d) and dw.weight.shape[0] == hidden:
                pad = dw.padding[0] if isinstance(dw.padding, tuple) else dw.padding
                local = nn.Conv1d(lh, lh, kernel_size=dw.kernel_size, groups=lh, padding=pad,
                                  bias=dw.bias is not None)
                with torch.no_grad():
                    local.weight.copy_(dw.weight.data[r * lh:(r + 1) * lh])
                    if dw.bias is not None:
                        local.bias.copy_(dw.bias.data[r * lh:(r + 1) * lh])
                conv.conv = local.to(dw.weight.device, dw.weight.dtype)
            n = _split(conv.out_proj.in_features, tp, "short-conv out_proj in")
            _shard_child(conv, "out_proj", col_offset=r * n, col_len=n)
            _install_input_copy(conv)
            handled.append("conv")
        ffn = getattr(layer, "feed_forward", None)
        if isinstance(ffn, nn.Module) and getattr(ffn, "w1", None) is not None:
            n = _split(ffn.w1.out_features, tp, "feed-forward intermediate")
            _shard_child(ffn, "w1", row_offset=r * n, row_len=n)
            _shard_child(ffn, "w3", row_offset=r * n, row_len=n)
            _shard_child(ffn, "w2", col_offset=r * n, col_len=n)
            _install_input_copy(ffn)
            handled.append("feed_forward")
        return handled

    @classmethod
    def gguf_name(cls, hf_name: str) -> Optional[str]:
        for pat, fmt in _GGUF_PATTERNS:
            m = pat.match(hf_name)
            if m:
                return fmt.format(*m.groups())
        return None  # the tied lm_head and unknown tensors

    @classmethod
    def transpose_embedding(cls) -> bool:
        return True
