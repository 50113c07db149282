"""Candidate-cache I/O on CPU: the exporter's cache reader
(reference voodoo_quant/tools/export_gguf.py:377-404) and arena packing from
memory-mapped cache files.  The staged host->HBM upload is covered by
tests/test_gpu_cache_io.py."""

from __future__ import annotations

import torch

from voodoo_quant import layers
from voodoo_quant.cache import arena_views, pack_arena
from voodoo_quant.quants import rtn
from voodoo_quant.tools.export_gguf import _load_cached_qbytes

TYPES = ["Q4_K", "Q6_K", "Q8_0"]


def _write_combined(root, name, w):
    d = root / name.removeprefix("model.").replace(".", "_")
    d.mkdir(parents=True)
    qb = {qt: rtn.quantize(w, qt) for qt in TYPES}
    torch.save(qb, d / f"combined_lazy_w{layers._tensor_hash(w)}_inone.pt")
    return qb


def test_export_reader_finds_cached_bytes(tmp_path, monkeypatch):
    monkeypatch.setattr(layers, "CANDIDATE_CACHE_DIR", tmp_path)
    torch.manual_seed(0)
    w = torch.randn(48, 512) * 0.02
    name = "model.layers.3.mlp.up_proj.weight"
    qb = _write_combined(tmp_path, name, w)
    for qt in TYPES:
        got = _load_cached_qbytes(name, qt, w)
        assert got is not None and got.dtype == torch.uint8 and got.shape[0] == 48
        assert torch.equal(got.reshape(-1), qb[qt].reshape(-1))
    assert _load_cached_qbytes(name, "Q5_K", w) is None  # type not cached
    assert _load_cached_qbytes(name, "Q4_K", w + 1e-3) is None  # other weight: other hash
    assert _load_cached_qbytes("model.layers.9.mlp.up_proj.weight", "Q4_K", w) is None
    (tmp_path / "layers_3_mlp_up_proj_weight" / f"combined_lazy_w{layers._tensor_hash(w)}_inone.pt").write_bytes(b"xx")
    assert _load_cached_qbytes(name, "Q4_K", w) is None  # unreadable file: fall back to quantising


def test_pack_arena_from_mmap(tmp_path):
    torch.manual_seed(1)
    w = torch.randn(64, 1024) * 0.02
    qb = {qt: rtn.quantize(w, qt) for qt in TYPES}
    p = tmp_path / "c.pt"
    torch.save(qb, p)
    mm = torch.load(p, weights_only=True, map_location="cpu", mmap=True)
    arena, layout = pack_arena(TYPES, [mm[qt] for qt in TYPES], 64, 1024, "cpu")
    assert all(l.offset % 256 == 0 for l in layout)
    for qt, v in zip(TYPES, arena_views(arena, layout)):
        assert torch.equal(v, qb[qt].reshape(v.shape))


def test_unreadable_or_short_cache_files_fail_loudly(tmp_path, monkeypatch):
    """Host-side faults in the candidate cache stop the layer's construction
    with an error that names the problem: a file that is not a torch file
    (RuntimeError naming the file), and a candidate of the wrong size for the
    tensor (ValueError with the expected and found sizes)."""
    import pytest

    monkeypatch.setattr(layers, "_CANDIDATE_CACHE_ROOT", tmp_path)
    w = torch.randn(16, 256) * 0.02
    path = layers._combined_cache_path("bad.proj", "lazy", layers._tensor_hash(w), "none")
    path.write_bytes(b"not a torch file" * 10)
    with pytest.raises(RuntimeError, match="cannot be read") as err:
        layers.MixedQuantLinear(256, 16, ["Q4_K"], w, tensor_name="bad.proj")
    assert str(path) in str(err.value)
    torch.save({"Q4_K": rtn.quantize(w, "Q4_K")[:-1]}, path)  # one block short
    with pytest.raises(ValueError, match="2160 != 2304"):
        layers.MixedQuantLinear(256, 16, ["Q4_K"], w, tensor_name="bad.proj")
