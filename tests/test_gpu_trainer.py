"""The full distillation step on the B200 kernels against a float32 torch
restatement of the reference step (voodoo_quant/training/trainer.py:
2443-2616): every gated weight is sum_k softmax(g / tau)_k * decode_k in
float32 (decoded by the CPU oracle) used through F.linear / F.embedding in a
float32 copy of the model; the loss is F.cross_entropy + T^2 * KL on its
float32 logits, plus the relu-squared size term.

The teacher is checked on its own first, against an independent path: every
weight quantised by the oracle's Q8_0 rule (oracle/q8_quant.py, pinned to
gguf-py), decoded by the oracle and used in float32 (F.linear / F.embedding
in an fp32 copy of the model): logits within 1e-2 relative.  The
restatement's KL then uses the step's own teacher logits, so the gate
gradients compare the student path alone.

Tolerances (bf16 operands with fp32 accumulation against float32): the loss
within 1e-2 relative; gate gradients of all tensors as one vector cosine >=
0.999 with relative L2 error < 3e-2; per tensor, cosine >= 0.999 with the
reference's default arguments, and >= 0.995 with the size term off (the
distillation gradient alone, a small difference signal between nearly equal
candidates, to which every bf16 rounding site of the step adds 1e-4 to 3e-4
of cosine).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from oracle import ggml_blocks, q8_quant

pytestmark = pytest.mark.gpu


class _TorchGated(nn.Module):
    def __init__(self, layer, embedding: bool):
        super().__init__()
        dev = layer.gates.device
        rows, pin, cols = layer.out_features, layer.padded_in_features, layer.in_features
        cands = []
        for qt, qb in zip(layer.candidate_types, layer._candidate_blocks()):
            w = ggml_blocks.dequantize(qb.cpu().numpy(), qt, rows, pin)[:, :cols]
            cands.append(torch.from_numpy(w).to(dev, torch.float32))
        self.cands = torch.stack(cands)
        self.gates = nn.Parameter(layer.gates.detach().clone())
        self.tau = layer.temperature
        self.embedding = embedding
        self.bpw = torch.tensor([ggml_blocks.FORMATS[q][2] / ggml_blocks.FORMATS[q][1]
                                 for q in layer.candidate_types], device=dev)
        self.numel = rows * cols

    def weight32(self):
        p = torch.softmax(self.gates / self.tau, dim=0)
        return torch.einsum("k,kij->ij", p, self.cands)

    def eff_bytes(self):
        return (torch.softmax(self.gates / self.tau, dim=0) * self.bpw).sum() * self.numel

    def forward(self, x):
        w = self.weight32()
        return F.embedding(x, w) if self.embedding else F.linear(x, w)


def _set(model, name, mod):
    parent = model
    *path, last = name.split(".")
    for p in path:
        parent = getattr(parent, p)
    setattr(parent, last, mod)


def _oracle_q8_teacher(shape, cuda, seed):
    """fp32 copy of the model whose every Linear / Embedding weight is the
    oracle's Q8_0 round trip of the bf16 weight."""
    from voodoo_quant.training import synthetic as S

    ref = S.build_llama(shape, cuda, seed=seed).float()
    for mod in ref.modules():
        if isinstance(mod, (nn.Linear, nn.Embedding)):
            w = mod.weight.detach().cpu().numpy()
            qb = q8_quant.quantize_q8_0(w)
            dec = ggml_blocks.dequantize(qb, "Q8_0", w.shape[0], w.shape[1])
            mod.weight.data = torch.from_numpy(dec).to(cuda)
    for p in ref.parameters():
        p.requires_grad = False
    return ref


# (distill_temperature, distill_weight, size_weight, size_tolerance), per-tensor cosine
_ARGS = {"default": ((1.0, 1.0, 10.0, 0.02), 0.999), "kd": ((2.0, 0.7, 0.0, 0.0), 0.995)}


@pytest.mark.parametrize("variant", ["default", "kd"])
def test_tiny_distill_step_matches_torch_restatement(cuda, variant):
    from voodoo_quant.layers import MixedQuantEmbedding
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    (Tk, kl_w, size_w, tol), per_tensor_cos = _ARGS[variant]
    args = StepArgs(distill_temperature=Tk, distill_weight=kl_w, size_weight=size_w, size_tolerance=tol)
    trainer, shape = build_distill("tiny", cuda, seed=3, args=args)
    # move the gates off zero so the softmax, the mixture and the size term are all non-trivial
    g = torch.Generator(device="cpu").manual_seed(5)
    with torch.no_grad():
        for layer in trainer.replaced.values():
            layer.gates.copy_(torch.randn(layer.num_candidates, generator=g).to(cuda))
    trainer.step_idx = 7
    x, y = S.random_tokens(shape, cuda, seed=11)

    # the step's teacher against the oracle's Q8_0 teacher in float32
    with torch.no_grad():
        t_logits = trainer.teacher(input_ids=x).logits.float()
        t_oracle = _oracle_q8_teacher(shape, cuda, seed=3)(input_ids=x).logits.float()
    assert float((t_logits - t_oracle).norm() / t_oracle.norm()) < 1e-2

    ref = S.build_llama(shape, cuda, seed=3).float()
    mods = {}
    for name, layer in trainer.replaced.items():
        mods[name] = _TorchGated(layer, isinstance(layer, MixedQuantEmbedding))
        _set(ref, name, mods[name])
    out = trainer.forward_backward(x, y)
    tau = out["tau"]
    for m in mods.values():
        m.tau = max(tau, 1e-6)
    for p in ref.parameters():
        p.requires_grad = False
    for m in mods.values():
        m.gates.requires_grad = True

    logits = ref(input_ids=x).logits.float()
    V = logits.shape[-1]
    T = args.distill_temperature
    lm = F.cross_entropy(logits.view(-1, V), y.view(-1))
    kl = F.kl_div(F.log_softmax(logits / T, -1).view(-1, V), F.softmax(t_logits / T, -1).view(-1, V),
                  reduction="none").sum(-1).mul(T * T).mean()
    cur = sum(m.eff_bytes() for m in mods.values()) + trainer.non_targeted_bytes
    size = torch.relu(torch.abs(cur / trainer.target_bytes - 1.0) - args.size_tolerance) ** 2
    loss = lm + args.distill_weight * kl + args.size_weight * size
    loss.backward()

    assert abs(out["loss"].item() - loss.item()) <= 1e-2 * abs(loss.item())
    assert abs(out["size_bytes"].item() - cur.item()) <= 1e-5 * cur.item()
    assert out["size_loss"].item() == pytest.approx(size.item(), rel=1e-4)
    ours = {n: trainer.replaced[n].gates.grad.double() for n in mods}
    theirs = {n: mods[n].gates.grad.double() for n in mods}
    per = {}
    for n in mods:
        assert torch.isfinite(ours[n]).all(), n
        per[n] = float(torch.dot(ours[n], theirs[n]) / (ours[n].norm() * theirs[n].norm()))
    assert min(per.values()) >= per_tensor_cos, per
    a, b = torch.cat([ours[n] for n in mods]), torch.cat([theirs[n] for n in mods])
    rel = (a - b).norm() / b.norm()
    cos = torch.dot(a, b) / (a.norm() * b.norm())
    assert rel < 3e-2 and cos > 0.999, (rel.item(), cos.item())


def test_tiny_distill_steps_reduce_loss_and_track_budget(cuda):
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    trainer, shape = build_distill("tiny", cuda, seed=0, args=StepArgs(max_steps=8))
    x, y = S.random_tokens(shape, cuda, seed=2)
    hist = [trainer.step(x, y) for _ in range(8)]
    assert all(torch.isfinite(h["loss"]) for h in hist)
    assert hist[-1]["tau"] == pytest.approx(0.01)
    # the uniform start (0.78 of the 8-bit bytes) is over the 0.45 budget; the size term drives the bytes down
    assert hist[-1]["size_bytes"].item() < hist[0]["size_bytes"].item()
    assert set(trainer.assignments().values()) <= set(shape.candidates)


@pytest.mark.parametrize("tied", [False, True])
def test_chunked_head_loss_equals_full_logits(cuda, tied):
    """--logits_chunk: head + loss per chunk of tokens (the last chunk ragged)
    gives the loss and gate gradients of the full-logits step (both with the
    token-count reduction).  Tolerance: loss 1e-5 relative; gate gradients
    1e-3 relative per tensor (the head's gate gradient is summed per chunk)."""
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    name = "tiny_tied" if tied else "tiny"
    if tied:
        base = S.SHAPES["tiny"]
        S.SHAPES[name] = S.ModelShape(base.layers, base.hidden, base.heads, base.kv_heads, base.ffn, base.vocab, True,
                                      candidates=list(base.candidates), batch=base.batch, seq=base.seq,
                                      budget=base.budget)
    out = {}
    for chunk in (0, 100):
        args = StepArgs(max_steps=4, ce_reduction="tokens", logits_chunk=chunk)
        trainer, shape = build_distill(name, cuda, seed=3, args=args)
        x, y = S.random_tokens(shape, cuda, seed=5)
        r = trainer.forward_backward(x, y)
        out[chunk] = (float(r["loss"]), float(r["lm_loss"]), float(r["distill_loss"]),
                      {n: m.gates.grad.detach().clone() for n, m in trainer.replaced.items()})
        del trainer
    a, b = out[0], out[100]
    for i in range(3):
        assert abs(a[i] - b[i]) <= 1e-5 * abs(a[i]) + 1e-7, (i, a[i], b[i])
    assert set(a[3]) == set(b[3])
    for n, g in a[3].items():
        h = b[3][n]
        assert float((g - h).norm()) <= 1e-3 * float(g.norm()) + 1e-9, n
