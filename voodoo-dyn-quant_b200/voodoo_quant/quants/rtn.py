"""Round-to-nearest GGUF block packer (a stand-in for libggml's quantisers).

The reference builds every candidate with llama.cpp's own quantiser
(libggml-base through ctypes, voodoo_quant/ggml.py:171-221).  That library is
not vendored and cannot be built offline, so seeded synthetic workloads and
tests need another source of *valid* packed blocks that approximate a given
weight matrix.  This module writes them with simple round-to-nearest rules:

* Q8_0 follows ggml's reference rule (d = amax/127, q = roundf(x/d)), which
  is also what gguf-py implements bit-exactly;
* the K-quants and IQ4_XS use per-sub-block RTN scales/minima quantised to
  the format's scale width, then RTN codes.  They are NOT byte-identical to
  llama.cpp's search-based quantisers (which are unavailable here); the byte
  layouts are exactly the GGUF structs, so the bit-exact decoders apply.

Works on any device (the benchmark quantises on the GPU).  Input: float
weights [rows, cols] with cols a multiple of 256 (32 for Q8_0).  Output:
uint8 [rows * cols / block_elems, block_bytes] on the same device.
"""

from __future__ import annotations

import torch

KVALUES_IQ4NL = (-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113)


def _roundf(v: torch.Tensor) -> torch.Tensor:
    """C roundf (half away from zero), exactly: floor(|v|) plus one when the
    fraction is at least 1/2 (floor(|v| + 0.5) would round 0.49999997 up)."""
    a = torch.abs(v)
    f = torch.floor(a)
    return torch.sign(v) * (f + torch.floor(2 * (a - f)))


def _f16_bytes(v: torch.Tensor) -> torch.Tensor:
    """float -> fp16 little-endian bytes [n, 2] uint8."""
    return v.to(torch.float16).contiguous().view(torch.uint8).reshape(-1, 2)


def _safe_div(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return torch.where(b != 0, a / torch.where(b != 0, b, torch.ones_like(b)), torch.zeros_like(a))


def _u8(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.int32).clamp(0, 255).to(torch.uint8)


def quantize_q8_0(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 32).float()
    d = x.abs().amax(dim=1, keepdim=True) / 127
    idv = torch.where(d == 0, torch.zeros_like(d), 1.0 / torch.where(d == 0, torch.ones_like(d), d))
    q = _roundf(x * idv).clamp(-127, 127).to(torch.int8).view(torch.uint8)
    return torch.cat([_f16_bytes(d.reshape(-1)), q], dim=1)


def _k4_pack_scales(sc: torch.Tensor, mn: torch.Tensor) -> torch.Tensor:
    """8 six-bit scales and mins -> the 12-byte Q4_K/Q5_K table."""
    sc = sc.to(torch.int32)
    mn = mn.to(torch.int32)
    out = torch.zeros(sc.shape[0], 12, dtype=torch.int32, device=sc.device)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return _u8(out)


def _affine_subblocks(x: torch.Tensor, nsub: int, qmax: int, sbits: int):
    """Per-sub-block scale/min (min <= 0 shifted to >= 0) quantised to sbits."""
    n = x.shape[0]
    xs = x.reshape(n, nsub, -1)
    lo = torch.clamp(xs.amin(dim=2), max=0.0)
    hi = xs.amax(dim=2)
    scale = (hi - lo) / qmax
    mins = -lo
    smax = (1 << sbits) - 1
    d = scale.amax(dim=1) / smax
    dmin = mins.amax(dim=1) / smax
    d16 = d.to(torch.float16).float()
    dm16 = dmin.to(torch.float16).float()
    sc = _roundf(_safe_div(scale, d16[:, None])).clamp(0, smax)
    mn = _roundf(_safe_div(mins, dm16[:, None])).clamp(0, smax)
    eff_s = d16[:, None] * sc
    eff_m = dm16[:, None] * mn
    q = _roundf(_safe_div(xs + eff_m[:, :, None], eff_s[:, :, None].expand_as(xs))).clamp(0, qmax)
    return d, dmin, sc, mn, q.reshape(n, -1).to(torch.int32)


def quantize_q4_k(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 256).float()
    d, dmin, sc, mn, q = _affine_subblocks(x, 8, 15, 6)
    q = q.reshape(-1, 4, 2, 32)
    qs = _u8(q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(-1, 128)
    return torch.cat([_f16_bytes(d), _f16_bytes(dmin), _k4_pack_scales(sc, mn), qs], dim=1)


def quantize_q5_k(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 256).float()
    d, dmin, sc, mn, q = _affine_subblocks(x, 8, 31, 6)
    q = q.reshape(-1, 8, 32)                                  # sub-block j, lane l
    qs = _u8((q[:, 0::2, :] & 15) | ((q[:, 1::2, :] & 15) << 4)).reshape(-1, 128)
    hi = (q >> 4) & 1                                          # bit j of qh[l]
    shifts = torch.arange(8, device=x.device, dtype=torch.int32).reshape(1, 8, 1)
    qh = _u8((hi << shifts).sum(dim=1))
    return torch.cat([_f16_bytes(d), _f16_bytes(dmin), _k4_pack_scales(sc, mn), qh, qs], dim=1)


def quantize_q6_k(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 256).float()
    n = x.shape[0]
    xs = x.reshape(n, 16, 16)
    scale = xs.abs().amax(dim=2) / 31
    d = scale.amax(dim=1) / 127
    d16 = d.to(torch.float16).float()
    sc = _roundf(_safe_div(scale, d16[:, None])).clamp(-128, 127)
    eff = (d16[:, None] * sc)[:, :, None].expand_as(xs)
    q = (_roundf(_safe_div(xs, eff)).clamp(-32, 31) + 32).to(torch.int32).reshape(n, 2, 4, 32)  # [h, g, l]
    ql = torch.stack([(q[:, :, 0] & 15) | ((q[:, :, 2] & 15) << 4),
                      (q[:, :, 1] & 15) | ((q[:, :, 3] & 15) << 4)], dim=2)                   # [n, h, 2, 32]
    qh = (q[:, :, 0] >> 4) | ((q[:, :, 1] >> 4) << 2) | ((q[:, :, 2] >> 4) << 4) | ((q[:, :, 3] >> 4) << 6)
    return torch.cat([_u8(ql).reshape(n, 128), _u8(qh).reshape(n, 64),
                      sc.to(torch.int8).view(torch.uint8).reshape(n, 16), _f16_bytes(d)], dim=1)


def _pack_2bit_k(q: torch.Tensor) -> torch.Tensor:
    """256 two-bit codes -> 64 bytes: element 128h + 32s + l at bits 2s of byte 32h + l."""
    n = q.shape[0]
    q = q.reshape(n, 2, 4, 32)
    shifts = (2 * torch.arange(4, device=q.device, dtype=torch.int32)).reshape(1, 1, 4, 1)
    return _u8(((q & 3) << shifts).sum(dim=2)).reshape(n, 64)


def quantize_q2_k(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 256).float()
    d, dmin, sc, mn, q = _affine_subblocks(x, 16, 3, 4)
    scales = _u8(sc.to(torch.int32) | (mn.to(torch.int32) << 4))
    return torch.cat([scales, _pack_2bit_k(q), _f16_bytes(d), _f16_bytes(dmin)], dim=1)


def quantize_q3_k(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 256).float()
    n = x.shape[0]
    xs = x.reshape(n, 16, 16)
    scale = xs.abs().amax(dim=2) / 4
    d = scale.amax(dim=1) / 31
    d16 = d.to(torch.float16).float()
    sc = _roundf(_safe_div(scale, d16[:, None])).clamp(0, 31)
    eff = (d16[:, None] * sc)[:, :, None].expand_as(xs)
    q = _roundf(_safe_div(xs, eff)).clamp(-4, 3).to(torch.int32).reshape(n, 256)
    high = (q >= 0).to(torch.int32)
    low = torch.where(q >= 0, q, q + 4)
    s6 = sc.to(torch.int32) + 32                                # stored value, signed scale + 32
    scb = torch.zeros(n, 12, dtype=torch.int32, device=x.device)
    for j in range(16):
        scb[:, j % 8] |= (s6[:, j] & 15) << (4 * (j // 8))
        scb[:, 8 + j % 4] |= ((s6[:, j] >> 4) & 3) << (2 * (j // 4))
    hb = high.reshape(n, 8, 32)                                 # bit b of hmask[l] = element 32b + l
    shifts = torch.arange(8, device=x.device, dtype=torch.int32).reshape(1, 8, 1)
    hmask = _u8((hb << shifts).sum(dim=1))
    return torch.cat([hmask, _pack_2bit_k(low), _u8(scb), _f16_bytes(d)], dim=1)


def quantize_iq4_xs(w: torch.Tensor) -> torch.Tensor:
    x = w.reshape(-1, 256).float()
    n = x.shape[0]
    xs = x.reshape(n, 8, 32)
    scale = xs.abs().amax(dim=2) / 127
    d = scale.amax(dim=1) / 31
    d16 = d.to(torch.float16).float()
    ls = _roundf(_safe_div(scale, d16[:, None])).clamp(0, 31)
    eff = (d16[:, None] * ls)[:, :, None].expand_as(xs)
    kv = torch.tensor(KVALUES_IQ4NL, dtype=torch.float32, device=x.device)
    v = _safe_div(xs, eff)
    q = (v[..., None] - kv).abs().argmin(dim=-1).to(torch.int32)  # [n, 8, 32]
    lsv = ls.to(torch.int32) + 32
    sl = _u8((lsv[:, 0::2] & 15) | ((lsv[:, 1::2] & 15) << 4))   # 4 bytes
    sh16 = (((lsv >> 4) & 3) << (2 * torch.arange(8, device=x.device, dtype=torch.int32))).sum(dim=1)
    sh = torch.stack([sh16 & 255, (sh16 >> 8) & 255], dim=1)
    qs = _u8(q[:, :, :16] | (q[:, :, 16:] << 4)).reshape(n, 128)
    return torch.cat([_f16_bytes(d), _u8(sh), sl, qs], dim=1)


QUANTIZERS = {
    "Q8_0": quantize_q8_0,
    "Q2_K": quantize_q2_k,
    "Q3_K": quantize_q3_k,
    "Q4_K": quantize_q4_k,
    "Q5_K": quantize_q5_k,
    "Q6_K": quantize_q6_k,
    "IQ4_XS": quantize_iq4_xs,
}


def quantize(weight: torch.Tensor, quant_type: str, row_chunk: int = 4096) -> torch.Tensor:
    """weight [rows, cols] -> packed uint8 [rows * cols / block_elems, block_bytes]."""
    if quant_type not in QUANTIZERS:
        raise ValueError(f"no round-to-nearest packer for {quant_type}; supported: {list(QUANTIZERS)}")
    be = 32 if quant_type == "Q8_0" else 256
    rows, cols = weight.shape
    if cols % be:
        raise ValueError(f"{quant_type} requires in_features % {be} == 0, got {cols}")
    parts = [QUANTIZERS[quant_type](weight[r:r + row_chunk]) for r in range(0, rows, row_chunk)]
    return torch.cat(parts, dim=0) if parts else torch.empty(0, dtype=torch.uint8, device=weight.device)
