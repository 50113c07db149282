"""Static-shape mode of the distillation step (``StepArgs(static_shapes=True)``,
``layers.set_static_shapes``): the host code of forward_backward makes no
device-to-host round trip and no data-dependent shape, so the step can be
recorded as one CUDA graph (``GatedDistillTrainer.capture``).  These CPU
tests check that the mode computes the same step, with the kernels replaced
by the torch stand-ins of tests/cpu_kernels.py:

* embedding lookups decode one row per token instead of the unique rows;
  the values are the same and the gate gradients equal up to the order of
  their float32 sums (1e-5 relative); the loss is bit-identical;
* the temperature is read from the gate bank's device scalar: the same
  float32 division, so the probabilities are bit-identical;
* under TP-2 (gloo), a vocabulary shard looks every token up at a clamped
  row and zeroes the others: same loss and gate gradients as the default
  TP step (1e-5 relative).
"""

from __future__ import annotations

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

pytest.importorskip("transformers")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shapes():
    from voodoo_quant.training import synthetic as S

    S.SHAPES["cpu_tp2"] = S.ModelShape(1, 512, 4, 2, 1024, 4096, False, head_dim=128,
                                       candidates=["Q4_K", "Q6_K", "Q8_0"], batch=2, seq=48, budget=0.45)


def _step(name: str, static: bool, tp: bool = False, step_idx: int = 3):
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    args = StepArgs(max_steps=8, ce_reduction="tokens", static_shapes=static, distill_temperature=1.5)
    trainer, shape = build_distill(name, "cpu", seed=3, args=args, tp=tp)
    from voodoo_quant import layers

    assert layers._STATIC_STATE.enabled == static
    g = torch.Generator().manual_seed(9)
    with torch.no_grad():
        for layer in trainer.replaced.values():
            layer.gates.copy_(torch.randn(layer.num_candidates, generator=g))
    trainer.step_idx = step_idx
    x, y = S.random_tokens(shape, "cpu", seed=5)
    out = trainer.forward_backward(x, y)
    assert (trainer.bank.tau_t is not None) == static
    probs = trainer.bank.probs().detach().clone()
    trainer.bank.release()
    grads = {n: m.gates.grad.detach().clone() for n, m in trainer.replaced.items()}
    return float(out["loss"]), float(out["size_bytes"]), grads, probs


def _close(a: dict, b: dict, rel: float) -> None:
    assert set(a) == set(b)
    for n in a:
        assert float((a[n] - b[n]).norm()) <= rel * float(b[n].norm()) + 1e-12, n


def test_static_step_equals_the_default_step():
    import cpu_kernels
    from voodoo_quant import layers

    undo = cpu_kernels.install()
    try:
        ref = _step("tiny", False)
        st = _step("tiny", True)
    finally:
        undo()
        layers.set_static_shapes(False)
    assert st[0] == ref[0] and st[1] == ref[1]
    assert torch.equal(st[3], ref[3])
    _close(st[2], ref[2], 1e-5)


def test_static_mode_requires_the_token_reduction():
    import cpu_kernels
    from voodoo_quant.training.trainer import StepArgs, build_distill

    undo = cpu_kernels.install()
    try:
        with pytest.raises(ValueError, match="tokens"):
            build_distill("tiny", "cpu", seed=3, args=StepArgs(static_shapes=True, ce_reduction="valid"))
    finally:
        undo()


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    import cpu_kernels
    from voodoo_quant import layers
    from voodoo_quant import parallel as P

    dist.init_process_group("gloo", rank=rank, world_size=world)
    _shapes()
    undo = cpu_kernels.install()
    try:
        P.adopt_process_group(0)
        res = {"default": _step("cpu_tp2", False, tp=True), "static": _step("cpu_tp2", True, tp=True)}
        torch.save(res, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        undo()
        layers.set_static_shapes(False)
        P.reset_tp()
        dist.destroy_process_group()


def test_static_tp2_step_equals_the_default_tp2_step():
    world = 2
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_worker, args=(world, _free_port(), td), nprocs=world, join=True, start_method="spawn")
        rs = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(world)]
    for r in rs:
        d, s = r["default"], r["static"]
        assert abs(s[0] - d[0]) <= 1e-6 * abs(d[0])
        assert s[1] == pytest.approx(d[1], rel=1e-9)
        _close(s[2], d[2], 1e-5)
