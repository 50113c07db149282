"""Host -> HBM upload of memory-mapped packed candidates through pinned
double-buffered staging (cache.pack_arena / cache.upload_staged): bytes land
unchanged, for tensors smaller than, equal to and larger than one staging
buffer, mixed with device-resident candidates."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_staged_upload_is_byte_exact(tmp_path):
    from voodoo_quant import cache
    from voodoo_quant.cache import arena_views, pack_arena

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(4)
    stage = cache._STAGE_BYTES
    sizes = [stage - 4096, stage, 2 * stage + 12345, 3 << 20]
    src = {f"t{i}": torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8) for i, n in enumerate(sizes)}
    p = tmp_path / "blobs.pt"
    torch.save(src, p)
    mm = torch.load(p, weights_only=True, map_location="cpu", mmap=True)
    dst = torch.zeros(sum(sizes) + 4096, dtype=torch.uint8, device=dev)
    pieces, off = [], 0
    for k in src:
        pieces.append((off, mm[k]))
        off += (mm[k].numel() + 255) // 256 * 256
    assert cache.upload_staged(dst, pieces) == sum(sizes)
    torch.cuda.synchronize()
    host = dst.cpu()
    for (o, t) in pieces:
        assert torch.equal(host[o:o + t.numel()], t)

    # pack_arena: host (mmap) candidates staged, a device candidate copied directly
    from voodoo_quant.quants import rtn

    w = torch.randn(2048, 4096, generator=g) * 0.02
    types = ["Q4_K", "Q6_K", "Q8_0"]
    qb = {qt: rtn.quantize(w, qt) for qt in types}
    torch.save(qb, tmp_path / "c.pt")
    mm = torch.load(tmp_path / "c.pt", weights_only=True, map_location="cpu", mmap=True)
    parts = [mm["Q4_K"], qb["Q6_K"].to(dev), mm["Q8_0"]]
    arena, layout = pack_arena(types, parts, 2048, 4096, dev)
    for qt, v in zip(types, arena_views(arena, layout)):
        assert torch.equal(v.cpu(), qb[qt].reshape(v.shape))
