"""Torch/numpy stand-ins for the CUDA kernels the training step calls --
TEST INFRASTRUCTURE ONLY.

``install()`` swaps the functions of ``voodoo_quant._C`` that the gated
layers, the Q8_0 teacher and the losses call for CPU implementations (block
decoding through ``oracle.ggml_blocks``, fp32 matmuls, a row-wise CE + KL),
so the host logic of the step -- the trainer, the gate bank, tensor
parallelism over gloo, the deferred gate-gradient queue, the chunked head
loss -- runs on CPU.  The stand-ins are consistent with one another, not
with the kernels' exact rounding; the kernels themselves are checked by the
GPU tests.  Returns an undo function.

``install(precision="bf16")`` (the default) rounds operands and results to
bf16 where the kernels do.  ``install(precision="fp32")`` keeps float32
operands and results, for float32 models, so that the step's host logic can
be compared with the reference's float32 step without bf16 rounding in the
way; a single-candidate decode (the Q8_0 teacher's weights) is still
rounded to bf16, as the reference's teacher does (dequantize_tensor_gpu,
voodoo_quant/layers.py:298-319).
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import ggml_blocks

# result dtype of the matmul / mixture / loss-gradient stand-ins (install())
_OUT = torch.bfloat16


def _decode(qb: torch.Tensor, qt: str, rows: int, cols: int) -> torch.Tensor:
    raw = qb.detach().cpu().contiguous().view(torch.uint8).numpy().reshape(-1)
    return torch.from_numpy(ggml_blocks.dequantize(raw, qt, rows, cols).astype(np.float32))


def _mix(qtypes, qbytes, probs, rows, padded_cols, cols, out=None):
    p = probs.detach().float().cpu().reshape(-1)
    w = torch.zeros(rows, padded_cols)
    for k, (qt, qb) in enumerate(zip(qtypes, qbytes)):
        w += p[k] * _decode(qb, qt, rows, padded_cols)
    ld = (cols + 7) // 8 * 8
    dt = torch.bfloat16 if len(qtypes) == 1 else _OUT
    res = torch.zeros(rows, ld, dtype=dt)
    res[:, :cols] = w[:, :cols].to(dt)
    if out is not None:
        out.copy_(res)
        return out
    return res


def _linear_fwd(x, w, n_out=None, in_features=None, out=None):
    kin = x.shape[1] if in_features is None else in_features
    n = w.shape[0] if n_out is None else n_out
    y = (x[:, :kin].float() @ w[:n, :kin].float().t()).to(_OUT)
    if out is not None:
        out.copy_(y)
        return out
    return y


def _linear_dx(dy, w, in_features, out=None):
    r = (dy.float() @ w[:, :in_features].float()).to(_OUT)
    if out is not None:
        out.copy_(r)
        return out
    return r


def _gategrad(dy, x, qtypes, qbytes, n_out, in_features, padded_cols, workspace=None, out=None):
    dw = dy.float().t() @ x[:, :in_features].float()
    g = torch.stack([(dw * _decode(qb, qt, n_out, padded_cols)[:, :in_features]).sum()
                     for qt, qb in zip(qtypes, qbytes)])
    if out is not None:
        out.copy_(g)
        return out
    return g


def _gategrad_grouped(dy, x, qtypes, qbytes_per_layer, rows, in_features, padded_cols, workspace=None, out=None):
    g, a = [], 0
    for n, qbytes in zip(rows, qbytes_per_layer):
        g.append(_gategrad(dy[:, a:a + n], x, qtypes, qbytes, n, in_features, padded_cols))
        a += n
    g = torch.stack(g)
    if out is not None:
        out.copy_(g)
        return out
    return g


def _dequant(qb, qt, rows, cols):
    return _decode(qb, qt, rows, cols)


def _row_lse(z: torch.Tensor) -> torch.Tensor:
    return torch.logsumexp(z, dim=1)


def _loss_fused(s, t, targets, temperature, ce_weight, kl_weight, want_grad=True):
    s, t, y = s.float(), t.float(), targets.long()
    T = float(temperature)
    valid = y >= 0
    lse = _row_lse(s)
    tgt = torch.where(valid, s.gather(1, y.clamp_min(0)[:, None])[:, 0], torch.zeros_like(lse))
    ce = torch.where(valid, lse - tgt, torch.zeros_like(lse))
    ls, lt = torch.log_softmax(s / T, 1), torch.log_softmax(t / T, 1)
    pt = lt.exp()
    kl = (pt * (lt - ls)).sum(1) * T * T
    g = None
    if want_grad:
        onehot = torch.zeros_like(s)
        onehot[valid, y[valid]] = 1.0
        g = (ce_weight * (torch.softmax(s, 1) - onehot) + kl_weight * T * (ls.exp() - pt)).to(_OUT)
    return ce, kl, g


def _loss_stats(s, t, targets, vocab_start, temperature):
    # per row: max / sum-exp of s, s/T and t/T on this shard, the cross term
    # sum exp(t/T - m) (t/T - s/T), and the target logit when it is on the shard
    s, t, y = s.float(), t.float(), targets.long()
    T = float(temperature)
    st = torch.zeros(s.shape[0], 8)
    for j, z in enumerate((s, s / T, t / T)):
        m = z.max(1).values
        st[:, 2 * j] = m
        st[:, 2 * j + 1] = torch.exp(z - m[:, None]).sum(1)
    e = torch.exp(t / T - st[:, 4][:, None])
    st[:, 6] = (e * (t / T - s / T)).sum(1)
    local = y - vocab_start
    on = (y >= 0) & (local >= 0) & (local < s.shape[1])
    st[:, 7] = torch.where(on, s.gather(1, local.clamp(0, s.shape[1] - 1)[:, None])[:, 0], torch.zeros(s.shape[0]))
    return st


def _loss_combine(stats, temperature):
    T = float(temperature)
    lse = torch.zeros(stats.shape[1], 4)
    for j in range(3):
        m = stats[:, :, 2 * j].max(0).values
        z = (stats[:, :, 2 * j + 1] * torch.exp(stats[:, :, 2 * j] - m)).sum(0)
        lse[:, j] = m + torch.log(z)
    mt = stats[:, :, 4].max(0).values
    zt = (stats[:, :, 5] * torch.exp(stats[:, :, 4] - mt)).sum(0)
    cross = (stats[:, :, 6] * torch.exp(stats[:, :, 4] - mt)).sum(0) / zt
    ce = lse[:, 0] - stats[:, :, 7].sum(0)
    kl = (cross - lse[:, 2] + lse[:, 1]) * T * T
    return lse, ce, kl


def _loss_grad(s, t, targets, vocab_start, temperature, row_lse, ce_weight, kl_weight):
    s, t, y = s.float(), t.float(), targets.long()
    T = float(temperature)
    local = y - vocab_start
    on = (y >= 0) & (local >= 0) & (local < s.shape[1])
    onehot = torch.zeros_like(s)
    onehot[on, local[on]] = 1.0
    valid = (y >= 0).float()[:, None]
    g = ce_weight * valid * (torch.exp(s - row_lse[:, 0:1]) - onehot) + kl_weight * T * (
        torch.exp(s / T - row_lse[:, 1:2]) - torch.exp(t / T - row_lse[:, 2:3]))
    return g.to(_OUT)


def _route_prep(keys, K):
    k = keys.to(torch.int64).reshape(-1).clamp(max=K - 1)
    order = torch.argsort(k, stable=True)
    inv = torch.empty_like(order)
    inv[order] = torch.arange(order.numel())
    off = torch.zeros(K + 1, dtype=torch.int32)
    off[1:] = torch.cumsum(torch.bincount(k, minlength=K), 0).to(torch.int32)
    return order, inv, off


def _linear_fwd_grouped(x, ws, n_out, in_features, group_off, out=None):
    y = torch.empty(x.shape[0], n_out, dtype=_OUT) if out is None else out
    off = group_off.tolist()
    for g, w in enumerate(ws):
        a, b = off[g], off[g + 1]
        if b > a:
            y[a:b] = _linear_fwd(x[a:b], w, n_out, in_features)
    return y


def _as_operand_fp32(x: torch.Tensor) -> torch.Tensor:
    return x if x.stride(-1) == 1 else x.contiguous()


def install(precision: str = "bf16"):
    global _OUT
    from voodoo_quant import _C
    from voodoo_quant.layers import _MixedQuantBase

    if precision not in ("bf16", "fp32"):
        raise ValueError(f"precision must be 'bf16' or 'fp32', got {precision!r}")
    prev_out = _OUT
    _OUT = torch.bfloat16 if precision == "bf16" else torch.float32
    table = [(_C, "mix", _mix), (_C, "linear_fwd", _linear_fwd), (_C, "linear_dx", _linear_dx),
             (_C, "gategrad", _gategrad), (_C, "dequant", _dequant), (_C, "loss_fused", _loss_fused),
             (_C, "route_prep", _route_prep), (_C, "linear_fwd_grouped", _linear_fwd_grouped),
             (_C, "loss_stats", _loss_stats), (_C, "loss_combine", _loss_combine), (_C, "loss_grad", _loss_grad),
             (_C, "gategrad_workspace_bytes", lambda n, k, c: 4),
             (_C, "gategrad_grouped", _gategrad_grouped),
             (_C, "gategrad_grouped_workspace_bytes", lambda n, k, g, c: 4),
             (_C, "set_gategrad_sm_reserve", lambda n: None), (_C, "set_gemm_sm_reserve", lambda n: None),
             (_MixedQuantBase, "_gategrad_workspace", lambda self, dev: None)]
    if precision == "fp32":
        table.append((_C, "_as_operand", _as_operand_fp32))
    saved = []
    for obj, name, fn in table:
        saved.append((obj, name, obj.__dict__.get(name), name in obj.__dict__))
        setattr(obj, name, fn)

    def undo():
        global _OUT
        _OUT = prev_out
        for obj, name, old, had in reversed(saved):
            if had:
                setattr(obj, name, old)
            else:
                delattr(obj, name)
    return undo
