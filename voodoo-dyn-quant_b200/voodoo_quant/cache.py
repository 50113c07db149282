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
import threading
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
    staged = []
    for lay, qb in zip(layout, qbytes):
        src = qb.reshape(-1).to(dtype=torch.uint8)
        if arena.is_cuda and src.device.type == "cpu" and lay.nbytes >= _STAGE_MIN:
            staged.append((lay, src))
        else:
            arena[lay.offset:lay.offset + lay.nbytes].copy_(src, non_blocking=False)
    if staged:
        upload_staged(arena, [(lay.offset, src) for lay, src in staged])
    return arena, layout


# Host -> HBM upload of packed blocks that sit in host memory (typically the
# mmap of a combined_lazy cache file): pages are copied into one of two pinned
# staging buffers while the other one's asynchronous copy to the device runs,
# so reading the file (page faults included) overlaps the PCIe transfer and
# the copies run at pinned-memory speed instead of through pageable bounces.
_STAGE_BYTES = 64 << 20
_STAGE_MIN = 1 << 20
_stage_bufs: list[torch.Tensor] = []
_stage_lock = threading.Lock()  # one upload at a time owns the staging buffers


def _staging_buffers() -> list[torch.Tensor]:
    if not _stage_bufs:
        _stage_bufs.extend(torch.empty(_STAGE_BYTES, dtype=torch.uint8).pin_memory() for _ in range(2))
    return _stage_bufs


def upload_staged(dst: torch.Tensor, pieces: list[tuple[int, torch.Tensor]]) -> int:
    """Copy host uint8 tensors into the device tensor `dst` at byte offsets
    (`pieces` = [(offset, host tensor)]) through double-buffered pinned
    staging on a side stream; returns the bytes copied.  The caller's stream
    waits for the copies.  Thread-safe: concurrent calls take turns."""
    with _stage_lock:
        return _upload_staged(dst, pieces)


def _upload_staged(dst: torch.Tensor, pieces: list[tuple[int, torch.Tensor]]) -> int:
    bufs = _staging_buffers()
    dev = dst.device
    side = torch.cuda.Stream(device=dev)
    done = [None, None]
    i = total = 0
    for off, src in pieces:
        src = src.reshape(-1)
        n = src.numel()
        for a in range(0, n, _STAGE_BYTES):
            b = i & 1
            if done[b] is not None:
                done[b].synchronize()  # the copy that last read this buffer has finished
            m = min(_STAGE_BYTES, n - a)
            bufs[b][:m].copy_(src[a:a + m])
            with torch.cuda.stream(side):
                dst[off + a:off + a + m].copy_(bufs[b][:m], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(side)
            done[b] = ev
            i += 1
            total += m
    torch.cuda.current_stream(dev).wait_stream(side)
    for ev in done:
        if ev is not None:
            ev.synchronize()  # the staging buffers may be reused by the next call
    return total


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
