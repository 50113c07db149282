"""Host-side pieces of the distillation step: the annealing schedule, the
8-bit byte budget and the construction of the tiny synthetic student."""

from __future__ import annotations

import math

import pytest
import torch


def test_anneal_temperature_schedule():
    from voodoo_quant.training.trainer import anneal_temperature

    assert anneal_temperature(0, 50, 1.0, 0.01) == 1.0
    assert math.isclose(anneal_temperature(49, 50, 1.0, 0.01), 0.01, rel_tol=1e-12)
    assert math.isclose(anneal_temperature(10, 50, 2.0, 0.5), 2.0 * 0.25 ** (10 / 49), rel_tol=1e-12)
    assert anneal_temperature(0, 1, 1.0, 0.01) == 0.01


def test_byte_budget_counts_shared_storage_once():
    from voodoo_quant.training.trainer import compute_non_targeted_8bit_bytes, compute_total_8bit_bytes

    meta = {"embed.weight": (100, 4096), "lm_head.weight": (100, 4096), "norm.weight": (200, 64),
            "q.weight": (300, 1024)}
    assert compute_total_8bit_bytes(meta) == 4096 + 64 + 1024
    # a storage is targeted if any key sharing it is
    assert compute_non_targeted_8bit_bytes(meta, {"embed.weight", "q.weight"}) == 64
    assert compute_non_targeted_8bit_bytes(meta, {"q.weight"}) == 4096 + 64


def test_build_tiny_distill_on_host():
    """The tiny synthetic student is built and accounted without a GPU."""
    pytest.importorskip("transformers")
    from voodoo_quant.training.q8_teacher import Q8Embedding, Q8Linear
    from voodoo_quant.training.trainer import build_distill

    trainer, shape = build_distill("tiny", "cpu", seed=0)
    names = set(trainer.replaced)
    assert "model.embed_tokens" in names and "lm_head" in names
    assert len(names) == 2 * 7 + 2
    params = 2 * (4 * 256 * 256 + 3 * 256 * 768 + 2 * 256) + 256 + 2 * 4096 * 256
    assert trainer.target_bytes == pytest.approx(shape.budget * params)
    assert trainer.non_targeted_bytes == 2 * 2 * 256 + 256  # the RMSNorm weights
    assert sum(p.requires_grad for p in trainer.student.parameters()) == len(names)
    assert isinstance(trainer.teacher.lm_head, Q8Linear)
    assert isinstance(trainer.teacher.model.embed_tokens, Q8Embedding)
    start = trainer.optimizer.param_groups[0]["lr"]
    assert start == 0.5
    with pytest.raises(RuntimeError, match="CUDA"):
        trainer.student(input_ids=torch.zeros(1, 4, dtype=torch.long))


def test_fused_blocks_leave_cpu_models_unchanged():
    """Patched modules run their original forward off the fused path (CPU here)."""
    pytest.importorskip("transformers")
    from voodoo_quant.fused_blocks import fuse_llama_blocks
    from voodoo_quant.training import synthetic as S

    shape = S.SHAPES["tiny"]
    a = S.build_llama(shape, "cpu", seed=2)
    b = S.build_llama(shape, "cpu", seed=2)
    assert fuse_llama_blocks(b) == 2 * 5 + 1  # per layer: two norms, attention, MLP, decoder add + norm
    x = torch.randint(0, shape.vocab, (1, 16))
    with torch.no_grad():
        assert torch.equal(a(input_ids=x, use_cache=False).logits, b(input_ids=x, use_cache=False).logits)
