"""numpy restatement of the distillation loss -- TEST INFRASTRUCTURE (oracle).

Reference: voodoo_quant/training/trainer.py:2567-2575 (plain path) and
:797-821 (token-chunked path); both compute, per token row with student
logits s, teacher logits t, target y and distillation temperature T,

    ce  = logsumexp(s) - s[y]
    kl  = T^2 * sum_v p_v (log p_v - log q_v),  p = softmax(t/T), q = softmax(s/T)

and return mean(ce) + lambda * mean(kl) (the chunked path uses lambda = 1 and
divides both sums by the token count).  The student-logit gradient is

    d/ds = [softmax(s) - onehot(y)] * ce_scale + lambda * T * (q - p) * kl_scale

with ce_scale = kl_scale = 1 / n_tokens.
"""

from __future__ import annotations

import numpy as np


def _lse(z: np.ndarray) -> np.ndarray:
    m = z.max(axis=-1, keepdims=True)
    return (m + np.log(np.exp(z - m).sum(axis=-1, keepdims=True)))[..., 0]


def row_terms(s: np.ndarray, t: np.ndarray, y: np.ndarray, temp: float):
    """Per-row (ce, kl) in float64; rows with y < 0 carry ce = 0."""
    s = np.asarray(s, np.float64)
    t = np.asarray(t, np.float64)
    lse = _lse(s)
    valid = y >= 0
    picked = np.where(valid, s[np.arange(s.shape[0]), np.clip(y, 0, s.shape[1] - 1)], 0.0)
    ce = np.where(valid, lse - picked, 0.0)
    lq = s / temp - _lse(s / temp)[:, None]
    lp = t / temp - _lse(t / temp)[:, None]
    p = np.exp(lp)
    kl = (p * (lp - lq)).sum(axis=-1) * temp * temp
    return ce, kl


def loss_and_grad(s: np.ndarray, t: np.ndarray, y: np.ndarray, temp: float, kl_weight: float = 1.0):
    """Chunked-path semantics: both sums divided by the token count."""
    n = s.shape[0]
    ce, kl = row_terms(s, t, y, temp)
    s64 = np.asarray(s, np.float64)
    t64 = np.asarray(t, np.float64)
    ps = np.exp(s64 - _lse(s64)[:, None])
    rows = np.nonzero(y >= 0)[0]
    ps[rows, y[rows]] -= 1.0
    ps[y < 0] = 0.0
    q = np.exp(s64 / temp - _lse(s64 / temp)[:, None])
    p = np.exp(t64 / temp - _lse(t64 / temp)[:, None])
    grad = (ps + kl_weight * temp * (q - p)) / n
    return ce.sum() / n, kl.sum() / n, grad
