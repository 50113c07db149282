"""numpy restatement of GGUF block decoding -- TEST INFRASTRUCTURE (oracle).

Every decoder returns float32 ``[nblocks, elems_per_block]`` from uint8
``[nblocks, block_bytes]`` and performs exactly the float32 operations of the
reference decoder it restates, in the same order, with no fused multiply-add
(numpy never contracts), so the results are bit-identical to the reference:

=========  ==========================================  =====================
format     reference decoder (file:line)               float32 op order
=========  ==========================================  =====================
Q8_0       voodoo_quant/layers.py:62-75                q * d
Q4_K       voodoo_quant/layers.py:78-122               (d*sc)*q - (dmin*m)
Q5_K       voodoo_quant/layers.py:125-179              (d*sc)*(q+16h) - (dmin*m)
Q6_K       voodoo_quant/layers.py:182-213              (d*sc)*(q-32)
IQ4_XS     voodoo_quant/quants/gpu_dequant.py:460-519  (d*(ls-32))*kvalue
Q2_K       gguf-py 0.19.0 quants.py Q2_K (no reference  (d*(sc&15))*q - (dmin*(sc>>4))
           decoder exists; registry lacks the type)
Q3_K       gguf-py 0.19.0 quants.py Q3_K (same)         (d*(sc-32))*q
=========  ==========================================  =====================

The byte layouts are the public GGUF block structs (ggml-common.h), which the
reference indexes by offset in the lines above.
"""

from __future__ import annotations

import numpy as np

QK_K = 256

# name -> (ggml type id, elements per block, bytes per block)
FORMATS = {
    "Q8_0": (8, 32, 34),
    "Q2_K": (10, 256, 84),
    "Q3_K": (11, 256, 110),
    "Q4_K": (12, 256, 144),
    "Q5_K": (13, 256, 176),
    "Q6_K": (14, 256, 210),
    "IQ4_XS": (23, 256, 136),
}

# IQ4_NL non-linear code book (public constant of the GGUF IQ4 formats).
KVALUES_IQ4NL = np.array(
    [-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113],
    dtype=np.float32,
)


def _f16(raw2: np.ndarray) -> np.ndarray:
    """Two little-endian bytes per row -> float32 (exact widening)."""
    return np.ascontiguousarray(raw2).view(np.float16).reshape(-1).astype(np.float32)


def _k4_scales(sc12: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Unpack the 12-byte 6-bit scale/min table of Q4_K/Q5_K.

    Restates ``get_scale_min_k4`` as unrolled in voodoo_quant/layers.py:91-105:
    j < 4:  sc = q[j] & 63,                      m = q[j+4] & 63
    j >= 4: sc = (q[j+4] & 15) | (q[j-4] >> 6) << 4,
            m  = (q[j+4] >> 4)  | (q[j]   >> 6) << 4
    """
    q = sc12.astype(np.int32)
    sc = np.empty((q.shape[0], 8), np.int32)
    mn = np.empty((q.shape[0], 8), np.int32)
    sc[:, :4] = q[:, 0:4] & 63
    mn[:, :4] = q[:, 4:8] & 63
    sc[:, 4:] = (q[:, 8:12] & 15) | ((q[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (q[:, 8:12] >> 4) | ((q[:, 4:8] >> 6) << 4)
    return sc.astype(np.float32), mn.astype(np.float32)


def dequant_q8_0(raw: np.ndarray) -> np.ndarray:
    """layers.py:62-75: y = int8(qs) * f16(d)."""
    d = _f16(raw[:, 0:2])
    qs = raw[:, 2:34].view(np.int8).astype(np.float32)
    return qs * d[:, None]


def dequant_q4_k(raw: np.ndarray) -> np.ndarray:
    """layers.py:78-122.  Block: d, dmin (f16), scales[12], qs[128]."""
    n = raw.shape[0]
    d = _f16(raw[:, 0:2])
    dmin = _f16(raw[:, 2:4])
    sc, mn = _k4_scales(raw[:, 4:16])
    qs = raw[:, 16:144].astype(np.int32)
    y = np.empty((n, QK_K), np.float32)
    for c in range(4):                       # 4 chunks of 64 weights
        q = qs[:, 32 * c:32 * c + 32]
        for half, nib in ((0, q & 15), (1, q >> 4)):
            j = 2 * c + half
            dl = d * sc[:, j]
            ml = dmin * mn[:, j]
            y[:, 32 * j:32 * j + 32] = dl[:, None] * nib.astype(np.float32) - ml[:, None]
    return y


def dequant_q5_k(raw: np.ndarray) -> np.ndarray:
    """layers.py:125-179.  Block: d, dmin, scales[12], qh[32], qs[128]."""
    n = raw.shape[0]
    d = _f16(raw[:, 0:2])
    dmin = _f16(raw[:, 2:4])
    sc, mn = _k4_scales(raw[:, 4:16])
    qh = raw[:, 16:48].astype(np.int32)
    qs = raw[:, 48:176].astype(np.int32)
    y = np.empty((n, QK_K), np.float32)
    for c in range(4):
        q = qs[:, 32 * c:32 * c + 32]
        for half, nib in ((0, q & 15), (1, q >> 4)):
            j = 2 * c + half                 # high bit j of qh[l]
            hi = ((qh >> j) & 1).astype(np.float32) * 16
            dl = d * sc[:, j]
            ml = dmin * mn[:, j]
            y[:, 32 * j:32 * j + 32] = dl[:, None] * (nib.astype(np.float32) + hi) - ml[:, None]
    return y


def dequant_q6_k(raw: np.ndarray) -> np.ndarray:
    """layers.py:182-213.  Block: ql[128], qh[64], scales[16] (int8), d (f16 last)."""
    n = raw.shape[0]
    ql = raw[:, 0:128].astype(np.int32)
    qh = raw[:, 128:192].astype(np.int32)
    sc = raw[:, 192:208].view(np.int8).astype(np.float32)
    d = _f16(raw[:, 208:210])
    y = np.empty((n, QK_K), np.float32)
    for h in range(2):                       # two halves of 128
        a = ql[:, 64 * h:64 * h + 32]
        b = ql[:, 64 * h + 32:64 * h + 64]
        hh = qh[:, 32 * h:32 * h + 32]
        quads = (
            (a & 15) | ((hh & 3) << 4),
            (b & 15) | (((hh >> 2) & 3) << 4),
            (a >> 4) | (((hh >> 4) & 3) << 4),
            (b >> 4) | (((hh >> 6) & 3) << 4),
        )
        for g, q in enumerate(quads):
            qf = q.astype(np.float32) - 32.0
            for part in range(2):            # scale index changes every 16
                si = 8 * h + part + 2 * g
                ds = d * sc[:, si]
                lo = 128 * h + 32 * g + 16 * part
                y[:, lo:lo + 16] = ds[:, None] * qf[:, 16 * part:16 * part + 16]
    return y


def dequant_q2_k(raw: np.ndarray) -> np.ndarray:
    """Q2_K, restating gguf-py 0.19.0 ``Q2_K.dequantize_blocks``.

    Block: scales[16] (low nibble scale, high nibble min), qs[64], d, dmin.
    Element e: half h = e // 128, shift s = (e % 128) // 32, l = e % 32,
    q = (qs[32h + l] >> 2s) & 3, sub-block e // 16.
    """
    n = raw.shape[0]
    scb = raw[:, 0:16].astype(np.int32)
    qs = raw[:, 16:80].astype(np.int32)
    d = _f16(raw[:, 80:82])
    dmin = _f16(raw[:, 82:84])
    dl = d[:, None] * (scb & 15).astype(np.float32)      # [n, 16]
    ml = dmin[:, None] * (scb >> 4).astype(np.float32)
    y = np.empty((n, QK_K), np.float32)
    for h in range(2):
        src = qs[:, 32 * h:32 * h + 32]
        for s in range(4):
            q = ((src >> (2 * s)) & 3).astype(np.float32)
            for part in range(2):
                e0 = 128 * h + 32 * s + 16 * part
                j = e0 // 16
                y[:, e0:e0 + 16] = dl[:, j:j + 1] * q[:, 16 * part:16 * part + 16] - ml[:, j:j + 1]
    return y


def q3k_scales(sc12: np.ndarray) -> np.ndarray:
    """16 signed 6-bit scales of Q3_K (value - 32), as int32 [n, 16].

    Scale j: low nibble from byte j % 8 (shifted by 4 for j >= 8), two high
    bits from byte 8 + j % 4 at shift 2 * (j // 4).
    """
    b = sc12.astype(np.int32)
    out = np.empty((b.shape[0], 16), np.int32)
    for j in range(16):
        lo = (b[:, j % 8] >> (4 * (j // 8))) & 15
        hi = (b[:, 8 + j % 4] >> (2 * (j // 4))) & 3
        out[:, j] = (lo | (hi << 4)) - 32
    return out


def dequant_q3_k(raw: np.ndarray) -> np.ndarray:
    """Q3_K, restating gguf-py 0.19.0 ``Q3_K.dequantize_blocks``.

    Block: hmask[32], qs[64], scales[12], d.  Element e: h = e // 128,
    s = (e % 128) // 32, l = e % 32; low bits (qs[32h + l] >> 2s) & 3, high
    bit (hmask[l] >> (e // 32)) & 1, value = low - 4 * (1 - high).
    """
    n = raw.shape[0]
    hm = raw[:, 0:32].astype(np.int32)
    qs = raw[:, 32:96].astype(np.int32)
    sc = q3k_scales(raw[:, 96:108]).astype(np.float32)
    d = _f16(raw[:, 108:110])
    dl = d[:, None] * sc                                   # [n, 16]
    y = np.empty((n, QK_K), np.float32)
    for h in range(2):
        src = qs[:, 32 * h:32 * h + 32]
        for s in range(4):
            e0 = 128 * h + 32 * s
            low = (src >> (2 * s)) & 3
            high = (hm >> (e0 // 32)) & 1
            q = (low - 4 * (high ^ 1)).astype(np.float32)
            for part in range(2):
                j = (e0 + 16 * part) // 16
                y[:, e0 + 16 * part:e0 + 16 * part + 16] = dl[:, j:j + 1] * q[:, 16 * part:16 * part + 16]
    return y


def dequant_iq4_xs(raw: np.ndarray) -> np.ndarray:
    """quants/gpu_dequant.py:460-519.  Block: d, scales_h (u16), scales_l[4], qs[128]."""
    n = raw.shape[0]
    d = _f16(raw[:, 0:2])
    sh = np.ascontiguousarray(raw[:, 2:4]).view(np.uint16).reshape(-1).astype(np.int32)
    sl = raw[:, 4:8].astype(np.int32)
    qs = raw[:, 8:136].astype(np.int32)
    y = np.empty((n, QK_K), np.float32)
    for ib in range(8):
        ls = ((sl[:, ib // 2] >> (4 * (ib % 2))) & 15) | (((sh >> (2 * ib)) & 3) << 4)
        dl = d * (ls.astype(np.float32) - 32.0)
        q = qs[:, 16 * ib:16 * ib + 16]
        y[:, 32 * ib:32 * ib + 16] = dl[:, None] * KVALUES_IQ4NL[q & 15]
        y[:, 32 * ib + 16:32 * ib + 32] = dl[:, None] * KVALUES_IQ4NL[q >> 4]
    return y


DECODERS = {
    "Q8_0": dequant_q8_0,
    "Q2_K": dequant_q2_k,
    "Q3_K": dequant_q3_k,
    "Q4_K": dequant_q4_k,
    "Q5_K": dequant_q5_k,
    "Q6_K": dequant_q6_k,
    "IQ4_XS": dequant_iq4_xs,
}


def dequantize(qbytes: np.ndarray, fmt: str, rows: int, cols: int) -> np.ndarray:
    """Packed row-major blocks -> float32 [rows, cols] (cols = padded width).

    Mirrors the contract of ``ggml.dequantize_tensor`` (ggml.py:224-269): the
    byte count must equal rows * cols / block_size * block_bytes.
    """
    _, bs, bb = FORMATS[fmt]
    if cols % bs:
        raise ValueError(f"{fmt} requires in_features % {bs} == 0, got {cols}")
    nb = rows * (cols // bs)
    flat = np.ascontiguousarray(qbytes, dtype=np.uint8).reshape(-1)
    if flat.size != nb * bb:
        raise ValueError(f"qweight size {flat.size} does not match {nb} blocks of {bb} bytes for {fmt}")
    return DECODERS[fmt](flat.reshape(nb, bb)).reshape(rows, cols)
