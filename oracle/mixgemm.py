"""numpy restatement of the gated-Linear arithmetic -- TEST INFRASTRUCTURE (oracle).

Reference semantics restated here (voodoo_quant/layers.py):

* probabilities   p = softmax(gates / tau), tau >= 1e-6          (:1342-1349)
* mixed weight    W_mix = sum_k p_k * W_k, W_k sliced to in_features (:336-352)
* forward         Y  = X W_mix^T                                  (:1730-1731)
* input grad      dX = dY W_mix                                   (autograd of F.linear)
* prob grad       g_k = <dY^T X, W_k> = sum_{o,i} (dY^T X)_{oi} W_k[o,i]  (:355-363)
* gate grad       dgates = (diag p - p p^T) g / tau               (softmax backward)
* assignment      argmax(gates), first maximum wins               (:1552-1557)

``fp64=True`` computes in float64 for a tighter reference; the default float32
matches the reference's own float32 CPU path.
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import ggml_blocks


def _row_chunks(n: int, parts: int):
    step = max(1, (n + parts - 1) // parts)
    return [(r, min(n, r + step)) for r in range(0, n, step)]


def softmax_probs(gates: np.ndarray, tau: float) -> np.ndarray:
    t = max(float(tau), 1e-6)
    z = np.asarray(gates, np.float64) / t
    z = z - z.max()
    e = np.exp(z)
    return (e / e.sum()).astype(np.float32)


def decode_candidates(blocks: list[np.ndarray], formats: list[str], rows: int, padded_cols: int,
                      cols: int, threads: int = 1) -> list[np.ndarray]:
    def one(bf):
        return ggml_blocks.dequantize(bf[0], bf[1], rows, padded_cols)[:, :cols]

    if threads <= 1:
        return [one(bf) for bf in zip(blocks, formats)]
    with ThreadPoolExecutor(threads) as ex:  # numpy ufuncs release the GIL
        return list(ex.map(one, zip(blocks, formats)))


def mixed_weight(cands: list[np.ndarray], probs: np.ndarray, fp64: bool = False, threads: int = 1) -> np.ndarray:
    """sum_k p_k W_k, accumulated in candidate order (row chunks run in parallel)."""
    dt = np.float64 if fp64 else np.float32
    w = np.empty(cands[0].shape, dt)

    def part(rng):
        r0, r1 = rng
        acc = w[r0:r1]
        acc[...] = 0
        for k, c in enumerate(cands):
            acc += dt(probs[k]) * c[r0:r1].astype(dt, copy=False)

    chunks = _row_chunks(w.shape[0], max(1, threads) * 4)
    if threads <= 1:
        for c in chunks:
            part(c)
    else:
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(part, chunks))
    return w


def linear_fwd(x: np.ndarray, w_mix: np.ndarray) -> np.ndarray:
    return x.astype(w_mix.dtype) @ w_mix.T


def linear_dx(dy: np.ndarray, w_mix: np.ndarray) -> np.ndarray:
    return dy.astype(w_mix.dtype) @ w_mix


def prob_grad(dy: np.ndarray, x: np.ndarray, cands: list[np.ndarray], fp64: bool = False,
              threads: int = 1) -> np.ndarray:
    """g_k = <dY^T X, W_k> (dW materialised, as in the reference)."""
    dt = np.float64 if fp64 else np.float32
    dw = dy.astype(dt, copy=False).T @ x.astype(dt, copy=False)
    return prob_grad_from_dw(dw, cands, threads=threads)


def prob_grad_from_dw(dw: np.ndarray, cands: list[np.ndarray], threads: int = 1) -> np.ndarray:
    """g_k = <dW, W_k> for a materialised dW (the reference's K reductions,
    voodoo_quant/layers.py:355-363), summed per row chunk in float64."""
    dt = dw.dtype
    chunks = _row_chunks(dw.shape[0], max(1, threads) * 4)

    def part(rng):
        r0, r1 = rng
        return [float(np.sum(dw[r0:r1] * c[r0:r1].astype(dt, copy=False), dtype=np.float64)) for c in cands]

    if threads <= 1:
        parts = [part(c) for c in chunks]
    else:
        with ThreadPoolExecutor(threads) as ex:
            parts = list(ex.map(part, chunks))
    return np.array(parts, np.float64).sum(axis=0)


def gate_grad(probs: np.ndarray, dprobs: np.ndarray, tau: float) -> np.ndarray:
    p = np.asarray(probs, np.float64)
    g = np.asarray(dprobs, np.float64)
    return (p * (g - np.dot(p, g))) / max(float(tau), 1e-6)


def assignment(gates: np.ndarray, candidate_types: list[str]) -> str:
    return candidate_types[int(np.argmax(np.asarray(gates)))]


def routed_linear_fwd(x: np.ndarray, cands: list[np.ndarray], routing: np.ndarray) -> np.ndarray:
    """PTQR forward y[t] = x[t] W_{routing[t]}^T in float32 (reference
    _RoutedMixedLinear.forward, voodoo_quant/layers.py:384-401).  Its
    backward is the mixture's: dX = dY W_mix, g_k = <dY^T X, W_k>."""
    y = np.zeros((x.shape[0], cands[0].shape[0]), np.float32)
    for k, w in enumerate(cands):
        rows = np.nonzero(routing == k)[0]
        if rows.size:
            y[rows] = x[rows].astype(np.float32) @ w.astype(np.float32).T
    return y


def bf16_round(a: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 (ties to even) -> float32; NaN stays NaN."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32)
    return np.where(np.isnan(a), np.float32(np.nan), out)


def routed_rows(rows_by_cand: list[np.ndarray], routing: np.ndarray) -> np.ndarray:
    """PTQR embedding rows: row i is candidate routing[i]'s decoded row,
    rounded to bf16 (reference _MixedEmbeddingRowFunctionLazy with routing,
    voodoo_quant/layers.py:702-728)."""
    out = np.zeros_like(rows_by_cand[0], dtype=np.float32)
    for k, r in enumerate(rows_by_cand):
        sel = routing == k
        out[sel] = r[sel]
    return bf16_round(out)
