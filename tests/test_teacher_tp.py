"""A teacher of its own TP degree (``StepArgs(teacher_tp=t)``), on CPU.

Under student TP-W the forward-only teacher can be sharded t ways inside
groups of t consecutive ranks, each group running it on its slice of the
batch; one all-to-all (``parallel.redistribute_vocab_shards``) then hands
every rank its vocabulary slice of all the teacher's logits.  Each teacher
all-reduce moves 1 / (W / t) of the tokens among t ranks instead of all of
them among W.

gloo, world size 4, kernels replaced by the torch stand-ins of
tests/cpu_kernels.py:
* the redistribution's index arithmetic, exactly, for t = 1, 2, 4 on
  logits whose values encode their global row and column;
* the TP-4 step with teacher_tp = 2 and 1 against the plain TP-4 step: the
  teacher's partial sums are split differently (over 2 or 1 ranks instead
  of 4), so the teacher logits differ by bf16 rounding only: loss within
  1e-3 relative, gate gradients cosine >= 0.999 per tensor.
"""

from __future__ import annotations

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

pytest.importorskip("transformers")

WORLD = 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _step(teacher_tp: int):
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    args = StepArgs(max_steps=8, ce_reduction="tokens", teacher_tp=teacher_tp, distill_temperature=1.5)
    trainer, shape = build_distill("cpu_tp4", "cpu", seed=3, args=args, tp=True)
    g = torch.Generator().manual_seed(9)
    with torch.no_grad():
        for layer in trainer.replaced.values():
            layer.gates.copy_(torch.randn(layer.num_candidates, generator=g))
    x, y = S.random_tokens(shape, "cpu", seed=5)
    out = trainer.forward_backward(x, y)
    grads = {n: m.gates.grad.detach().clone() for n, m in trainer.replaced.items()}
    return float(out["loss"]), grads


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    import cpu_kernels
    from voodoo_quant import parallel as P
    from voodoo_quant.training import synthetic as S

    dist.init_process_group("gloo", rank=rank, world_size=world)
    S.SHAPES["cpu_tp4"] = S.ModelShape(1, 512, 4, 4, 1024, 4096, False, head_dim=128, candidates=["Q4_K", "Q8_0"],
                                       batch=4, seq=24, budget=0.45)
    undo = cpu_kernels.install()
    try:
        P.adopt_process_group(0)
        res = {"redistribute": []}
        B, Sq, V = 4, 3, 16
        for t in (1, 2, 4):
            G = world // t
            g, h, b, Vt = rank // t, rank % t, B // G, V // t
            rows = torch.arange(g * b, (g + 1) * b).view(b, 1, 1)
            cols = torch.arange(h * Vt, (h + 1) * Vt).view(1, 1, Vt)
            local = (rows * 1000 + cols + torch.zeros(1, Sq, 1)).to(torch.bfloat16 if t == 2 else torch.float32)
            out = P.redistribute_vocab_shards(local, t)
            want = (torch.arange(B).view(B, 1, 1) * 1000 + torch.arange(rank * V // world, (rank + 1) * V // world)
                    .view(1, 1, -1) + torch.zeros(1, Sq, 1))
            # the all-to-all moves bits: compare with the expected values at the input's precision
            res["redistribute"].append(bool(out.dtype == local.dtype
                                            and torch.equal(out.float(), want.to(local.dtype).float())))
        res["plain"] = _step(0)
        res["t2"] = _step(2)
        res["t1"] = _step(1)
        torch.save(res, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        undo()
        P.reset_tp()
        dist.destroy_process_group()


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float(a @ b / (a.norm() * b.norm() + 1e-300))


def test_teacher_of_its_own_tp_degree_tp4():
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_worker, args=(WORLD, _free_port(), td), nprocs=WORLD, join=True, start_method="spawn")
        rs = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(WORLD)]
    for r in rs:
        assert r["redistribute"] == [True, True, True]
        plain = r["plain"]
        for key in ("t2", "t1"):
            loss, grads = r[key]
            assert abs(loss - plain[0]) <= 1e-3 * abs(plain[0]), (key, loss, plain[0])
            for n, g in plain[1].items():
                assert _cos(grads[n], g) >= 0.999, (key, n, _cos(grads[n], g))
    for key in ("plain", "t2", "t1"):  # every rank ends with the same (all-reduced) gate gradients
        for n in rs[0][key][1]:
            assert all(torch.equal(rs[0][key][1][n], rk[key][1][n]) for rk in rs[1:]), (key, n)
