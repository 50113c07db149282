"""Compile-cache setup and the HBM-resident packed-candidate store.

``setup_caches`` keeps the reference's import-time contract
(voodoo_quant/cache.py:1-24): Triton/Inductor cache directories inside the
project tree.

``PackedCandidateStore`` is the candidate cache of the B200 path.  The
reference keeps, per gated tensor, either K dequantised bf16 copies on the
host (non-lazy ``_w_k``, voodoo_quant/layers.py:1139-1143) or K packed byte
tensors that are re-dequantised on every forward and backward
(``_qweight_k``, :1136-1138, :480-667).  Here the K packed GGUF block streams
of a tensor live in ONE device allocation (an "arena"), each candidate at a
256-byte aligned offset, in the exact row-major block layout libggml writes
([rows * padded_cols / block_elems, block_bytes] uint8).  The gated-Linear
kernels read them in place; nothing dequantised is ever stored.

Sizing: bytes per weight for a candidate menu is sum_k block_bytes_k /
block_elems_k (e.g. Q2_K..Q8_0 = 3.8906 B/weight), so an 8B-shape model with
six candidates holds ~29 GB of packed blocks, well inside 180 GB of HBM.
"""

from __future__ import annotations

import os
import weakref
from dataclasses import dataclass
from pathlib import Path

import torch

_ROOT = Path(__file__).resolve().parent.parent


def setup_caches() -> None:
    os.environ.setdefault("TRITON_CACHE_DIR", str(_ROOT / ".triton_cache"))
    os.environ.setdefault("TORCHINDUCTOR_CACHE_DIR", str(_ROOT / ".torchinductor_cache"))
    os.environ.setdefault("TORCHINDUCTOR_COMPILE_THREADS", "1")
    for k in ("TRITON_CACHE_DIR", "TORCHINDUCTOR_CACHE_DIR"):
        try:
            Path(os.environ[k]).mkdir(parents=True, exist_ok=True)
        except OSError:
            pass


setup_caches()

_ALIGN = 256


@dataclass
class CandidateLayout:
    """Where candidate k of a tensor sits inside its arena."""

    qtype: str
    offset: int
    nbytes: int
    block_bytes: int


def pack_arena(types: list[str], qbytes: list[torch.Tensor], rows: int, padded_cols: int,
               device: torch.device | str, name: str = "tensor") -> tuple[torch.Tensor, list[CandidateLayout]]:
    """Copy K packed candidates into one device allocation (256-byte aligned slots)."""
    from voodoo_quant.ggml import get_quant_info

    if len(types) != len(qbytes):
        raise ValueError(f"{name}: {len(types)} candidate types but {len(qbytes)} byte tensors")
    layout, off = [], 0
    for qt, qb in zip(types, qbytes):
        info = get_quant_info(qt)
        if padded_cols % info.block_size:
            raise ValueError(f"{name}: {qt} needs in_features % {info.block_size} == 0, got {padded_cols}")
        expect = rows * (padded_cols // info.block_size) * info.block_bytes
        if qb.numel() != expect:
            raise ValueError(f"{name}: {qt} qbytes numel {qb.numel()} != {expect} for [{rows}x{padded_cols}]")
        layout.append(CandidateLayout(qt, off, expect, info.block_bytes))
        off += (expect + _ALIGN - 1) // _ALIGN * _ALIGN
    arena = torch.empty(max(off, _ALIGN), dtype=torch.uint8, device=device)
    for lay, qb in zip(layout, qbytes):
        arena[lay.offset:lay.offset + lay.nbytes].copy_(qb.reshape(-1).to(dtype=torch.uint8), non_blocking=False)
    return arena, layout


def arena_views(arena: torch.Tensor, layout: list[CandidateLayout]) -> list[torch.Tensor]:
    """[nblocks_k, block_bytes_k] views of each candidate inside the arena."""
    return [arena[l.offset:l.offset + l.nbytes].view(-1, l.block_bytes) for l in layout]


class PackedCandidateStore:
    """Process-wide index of the resident candidate arenas (name -> owner).

    Owners are the gated modules; the index holds weak references only, so
    deleting a module frees its HBM.  Used for accounting and lookup.
    """

    def __init__(self) -> None:
        self._owners: "weakref.WeakValueDictionary[str, object]" = weakref.WeakValueDictionary()

    def register(self, name: str, owner) -> None:
        self._owners[name] = owner

    def get(self, name: str):
        return self._owners.get(name)

    def __contains__(self, name: str) -> bool:
        return name in self._owners

    def __len__(self) -> int:
        return len(self._owners)

    def items(self):
        return list(self._owners.items())

    def total_bytes(self) -> int:
        total = 0
        for _, m in self.items():
            total += sum(l.nbytes for l in getattr(m, "_cand_layout", []))
        return total

    def clear(self) -> None:
        self._owners.clear()


STORE = PackedCandidateStore()
