"""Q8_0 quantisation, CPU restatement -- TEST INFRASTRUCTURE ONLY.

The reference quantises through libggml (``ggml.quantize_tensor``,
voodoo_quant/ggml.py:171-221; the Q8_0 teacher, training/q8_teacher.py).  For
Q8_0 the rule is ggml's reference ``quantize_row_q8_0``, which gguf-py 0.19.0
(the reference's declared dependency) restates bit-exactly in
``gguf/quants.py`` ``Q8_0.quantize_blocks``; ``tests/golden/q8quant_golden.npz``
holds gguf-py's output and pins this restatement.  Per 32-element block:

    d  = max |x| / 127          (float32)
    id = 1 / d, or 0 when d == 0 (float32)
    q  = round half away from zero (x * id), as int8
    block = fp16(d) little-endian, then the 32 codes.
"""

from __future__ import annotations

import numpy as np


def roundf(v: np.ndarray) -> np.ndarray:
    """C roundf on float32: floor(|v|), plus one when the fraction is >= 1/2."""
    a = np.abs(v)
    f = np.floor(a)
    return np.sign(v) * (f + np.floor(2 * (a - f)))


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """float32 [rows, cols] (cols % 32 == 0) -> uint8 [rows * cols / 32, 34]."""
    x = np.ascontiguousarray(w, dtype=np.float32).reshape(-1, 32)
    d = (np.abs(x).max(axis=1, keepdims=True) / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d == 0, np.float32(0), (np.float32(1) / d)).astype(np.float32)
    q = roundf((x * idv).astype(np.float32)).astype(np.int8)
    return np.concatenate([d.astype(np.float16).view(np.uint8), q.view(np.uint8)], axis=1)
