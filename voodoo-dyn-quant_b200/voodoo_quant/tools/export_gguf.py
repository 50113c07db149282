"""Candidate-cache reader of the GGUF exporter (reference
voodoo_quant/tools/export_gguf.py:377-404).

Only the part of the exporter that reads the packed candidate store is on
this path: an export reuses the llama.cpp-quantised bytes the training step
cached (``combined_lazy_w{hash}_inone.pt``, one uint8 [nblocks, block_bytes]
tensor per type, memory-mapped) instead of re-running the quantiser.  The
rest of the exporter (GGUF writing, metadata, tokenizer) is tooling outside
the training step.
"""

from __future__ import annotations

import torch

from voodoo_quant import layers
from voodoo_quant.ggml import get_quant_info


def _load_cached_qbytes(hf_name: str, quant_type: str, weight: torch.Tensor) -> torch.Tensor | None:
    """Cached packed bytes of (hf tensor name, quant type) as a [out_features,
    row bytes] uint8 view of the memory-mapped cache file, or None when that
    exact weight (by content hash) and type are not cached.  Any read error
    also gives None: the caller then quantises from the weight."""
    try:
        stripped = hf_name.removeprefix("model.")
        weight_hash = layers._tensor_hash(weight)
        p = layers.CANDIDATE_CACHE_DIR / stripped.replace(".", "_") / f"combined_lazy_w{weight_hash}_inone.pt"
        if not p.exists():
            return None
        combined = torch.load(p, weights_only=True, map_location="cpu", mmap=True)
        qb = combined.get(quant_type)
        if qb is None:
            return None
        get_quant_info(quant_type)  # unknown type -> error -> None
        return qb.reshape(weight.shape[0], -1)
    except Exception:
        return None


load_cached_qbytes = _load_cached_qbytes
