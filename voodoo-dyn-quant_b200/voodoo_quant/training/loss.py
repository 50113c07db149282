"""Fused CE + lambda * T^2 * KL(teacher || student) on the B200 loss kernel.

Replaces the reference's loss blocks (voodoo_quant/training/trainer.py):

* plain path :2567-2575  -- ``distillation_loss(..., ce_reduction="valid")``:
  mean CE over non-ignored tokens (F.cross_entropy's default, ignore id -100)
  plus ``distill_weight`` * mean per-token T^2 * KL;
* chunked path :797-821 -- ``ce_reduction="tokens"``: both sums divided by
  the token count;
* head-chunked path :753-832 -- ``chunked_head_loss``: the student and teacher
  heads run per token chunk on the final hidden states, each chunk's loss is
  back-propagated through the head at once, so no [tokens, V] logits tensor
  ever exists (peak: one chunk's logits and gradient);
* vocab-parallel path :915-1066 -- ``tp_distillation_loss``: each rank holds
  the logits of its vocabulary shard; per-row partial statistics from one
  pass over the shard are all-gathered once (one collective, instead of the
  reference's MAX + SUM + SUM per token chunk), combined, and the gradient is
  written for the local shard.

The kernel reads student and teacher logits once for the statistics and once
more (L2-resident) for the gradient, which it writes in bf16; the returned
loss is a scalar whose backward scales that stored gradient.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch.autograd import Function

from voodoo_quant import _C


def _weights(targets: torch.Tensor, n: int, distill_weight: float, ce_reduction: str):
    if ce_reduction == "valid":
        n_valid = int((targets >= 0).sum().item()) if targets.numel() else 0
        ce_w = 1.0 / max(n_valid, 1)
    elif ce_reduction == "tokens":
        ce_w = 1.0 / max(n, 1)
    else:
        raise ValueError(f"ce_reduction must be 'valid' or 'tokens', got {ce_reduction!r}")
    return ce_w, distill_weight / max(n, 1)


def _scaled(g: torch.Tensor, g_loss: torch.Tensor, unit: bool) -> torch.Tensor:
    """The stored logits gradient times the loss's upstream gradient; with
    ``unit`` the caller seeds the loss with 1 (``loss.backward()`` on a sum
    in which the loss has coefficient 1), so the [tokens, V] gradient is
    returned as it is instead of being multiplied by 1 in another pass."""
    return g if unit else g * g_loss.to(g.dtype)


class _FusedDistillLoss(Function):
    @staticmethod
    def forward(ctx, s: torch.Tensor, t: torch.Tensor, y: torch.Tensor, temperature: float, ce_w: float,
                kl_w: float, unit_upstream: bool = False):
        need = s.requires_grad
        ce, kl, g = _C.loss_fused(s, t, y, temperature, ce_w, kl_w, want_grad=need)
        ctx.g = g
        ctx.unit = unit_upstream
        ctx.s_dtype = s.dtype
        ce_sum, kl_sum = ce.sum(), kl.sum()
        ctx.mark_non_differentiable(ce_sum, kl_sum)
        return ce_w * ce_sum + kl_w * kl_sum, ce_sum, kl_sum

    @staticmethod
    def backward(ctx, g_loss, _g_ce, _g_kl):
        g = ctx.g
        ctx.g = None
        if g is None:
            return None, None, None, None, None, None, None
        return _scaled(g, g_loss, ctx.unit).to(ctx.s_dtype), None, None, None, None, None, None


def distillation_loss(student_logits: torch.Tensor, teacher_logits: torch.Tensor, targets: torch.Tensor,
                      temperature: float = 1.0, distill_weight: float = 1.0, ce_reduction: str = "valid",
                      unit_upstream: bool = False):
    """Returns (loss, lm_loss, distill_loss) like the reference's plain path.

    ``loss = lm_loss + distill_weight * distill_loss`` is differentiable with
    respect to ``student_logits`` ([..., V]); lm_loss / distill_loss are
    detached scalars (mean CE, mean per-token T^2 * KL).  ``unit_upstream``:
    the caller back-propagates with gradient 1 into ``loss`` (see ``_scaled``).
    """
    V = student_logits.shape[-1]
    s = student_logits.reshape(-1, V)
    t = teacher_logits.reshape(-1, V).detach()
    y = targets.reshape(-1)
    n = s.shape[0]
    ce_w, kl_w = _weights(y, n, distill_weight, ce_reduction)
    loss, ce_sum, kl_sum = _FusedDistillLoss.apply(s, t, y, float(temperature), ce_w, kl_w, bool(unit_upstream))
    return loss, (ce_sum * ce_w).detach(), (kl_sum / max(n, 1)).detach()


class _TPFusedDistillLoss(Function):
    @staticmethod
    def forward(ctx, s, t, y, vocab_start, temperature, ce_w, kl_w, group, unit_upstream=False):
        stats = _C.loss_stats(s, t, y, vocab_start, temperature)            # [rows, 8]
        world = dist.get_world_size(group)
        # [world * rows, 8], viewed per rank: gloo wants the ranks stacked along dim 0
        gathered = torch.empty((world * stats.shape[0],) + tuple(stats.shape[1:]), dtype=stats.dtype,
                               device=stats.device)
        dist.all_gather_into_tensor(gathered, stats, group=group)
        gathered = gathered.view((world,) + tuple(stats.shape))
        lse, ce, kl = _C.loss_combine(gathered, temperature)
        ctx.g = _C.loss_grad(s, t, y, vocab_start, temperature, lse, ce_w, kl_w) if s.requires_grad else None
        ctx.unit = unit_upstream
        ctx.s_dtype = s.dtype
        ce_sum, kl_sum = ce.sum(), kl.sum()
        ctx.mark_non_differentiable(ce_sum, kl_sum)
        return ce_w * ce_sum + kl_w * kl_sum, ce_sum, kl_sum

    @staticmethod
    def backward(ctx, g_loss, _a, _b):
        g = ctx.g
        ctx.g = None
        if g is None:
            return (None,) * 9
        return _scaled(g, g_loss, ctx.unit).to(ctx.s_dtype), None, None, None, None, None, None, None, None


def tp_distillation_loss(student_shard: torch.Tensor, teacher_shard: torch.Tensor, targets: torch.Tensor,
                         vocab_start: int, temperature: float = 1.0, distill_weight: float = 1.0,
                         ce_reduction: str = "tokens", group=None, unit_upstream: bool = False):
    """Vocabulary-parallel loss: every rank passes its [..., V/N] logits shard.

    The returned loss is the exact global loss on every rank; its gradient
    covers this rank's shard only (each rank differentiates its own logits).
    """
    V = student_shard.shape[-1]
    s = student_shard.reshape(-1, V)
    t = teacher_shard.reshape(-1, V).detach()
    y = targets.reshape(-1)
    n = s.shape[0]
    ce_w, kl_w = _weights(y, n, distill_weight, ce_reduction)
    loss, ce_sum, kl_sum = _TPFusedDistillLoss.apply(s, t, y, int(vocab_start), float(temperature), ce_w, kl_w,
                                                     group, bool(unit_upstream))
    return loss, (ce_sum * ce_w).detach(), (kl_sum / max(n, 1)).detach()


def chunked_head_loss(student_head, teacher_head, hidden: torch.Tensor, t_hidden: torch.Tensor,
                      targets: torch.Tensor, chunk: int, temperature: float = 1.0, distill_weight: float = 1.0,
                      vocab_start: int | None = None, group=None):
    """Head + loss per token chunk (reference ``_chunked_forward_loss``,
    voodoo_quant/training/trainer.py:753-832).

    ``hidden`` / ``t_hidden`` are the final hidden states of the student and
    teacher stacks ([..., H]); for each chunk of ``chunk`` tokens the student
    head (gated or plain) and the teacher head produce that chunk's logits,
    the fused kernel gives its CE + T^2 * KL and logit gradient, and the
    chunk's loss is back-propagated through the student head immediately
    (the head's gate gradients accumulate over the chunks).  Both terms are
    token sums divided by the token count (``ce_reduction="tokens"``), so the
    chunked loss equals the unchunked one.  With ``vocab_start`` the heads
    are vocabulary-parallel shards and each chunk uses the TP loss.

    Returns (grad of ``hidden`` [same shape, detached], loss, lm_loss,
    distill_loss) with detached scalars; the caller back-propagates the
    hidden-state gradient through the stack once.
    """
    if chunk <= 0:
        raise ValueError(f"chunk must be positive, got {chunk}")
    H = hidden.shape[-1]
    s_flat = hidden.detach().reshape(-1, H)
    t_flat = t_hidden.detach().reshape(-1, H)
    y_flat = targets.reshape(-1)
    n = s_flat.shape[0]
    ce_w, kl_w = _weights(y_flat, n, distill_weight, "tokens")
    h_grad = torch.zeros_like(s_flat)
    loss = torch.zeros((), dtype=torch.float32, device=s_flat.device)
    ce_tot = torch.zeros((), dtype=torch.float32, device=s_flat.device)
    kl_tot = torch.zeros((), dtype=torch.float32, device=s_flat.device)
    for i in range(0, n, chunk):
        h_c = s_flat[i:i + chunk].requires_grad_(True)
        s_c = student_head(h_c)
        with torch.no_grad():
            t_c = teacher_head(t_flat[i:i + chunk])
        y_c = y_flat[i:i + chunk]
        V = s_c.shape[-1]
        if vocab_start is not None:
            loss_c, ce_c, kl_c = _TPFusedDistillLoss.apply(s_c.reshape(-1, V), t_c.reshape(-1, V).detach(), y_c,
                                                           int(vocab_start), float(temperature), ce_w, kl_w, group,
                                                           True)
        else:
            loss_c, ce_c, kl_c = _FusedDistillLoss.apply(s_c.reshape(-1, V), t_c.reshape(-1, V).detach(), y_c,
                                                         float(temperature), ce_w, kl_w, True)
        del t_c
        loss_c.backward()
        if h_c.grad is not None:
            h_grad[i:i + chunk] = h_c.grad
        loss = loss + loss_c.detach()
        ce_tot = ce_tot + ce_c
        kl_tot = kl_tot + kl_c
        del s_c, loss_c, h_c
    return h_grad.reshape(hidden.shape), loss, (ce_tot * ce_w).detach(), (kl_tot / max(n, 1)).detach()
