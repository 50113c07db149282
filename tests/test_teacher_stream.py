"""The teacher's forward on a stream of its own (``StepArgs(teacher_stream=True)``).

Under TP the teacher's row-parallel sums then go to a communicator of their
own (``parallel.enable_teacher_overlap``, ``parallel.collectives_on``), so
they can run while the student's kernels run on the main stream.  On CPU
(gloo, world size 2, host stand-ins for the CUDA streams and the torch
stand-ins of tests/cpu_kernels.py for the kernels) this checks the wiring:
the step is bit for bit the default step (with the head + loss per token
chunk, equal up to the order of its sums), the teacher's forward collectives all go to the teacher's
communicator, the student's stay on the TP group, and with an SM reserve
the forward GEMMs leave it free while both forwards are issued and not
after.
"""

from __future__ import annotations

import contextlib
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


class _Stream:
    def wait_stream(self, other):
        pass


def _host_streams():
    torch.cuda.Stream = _Stream
    torch.cuda.current_stream = lambda *a, **k: _Stream()
    torch.cuda.stream = lambda s: contextlib.nullcontext()


def _step(teacher_stream: bool, chunk: int, log: list, sms: int = 0):
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    args = StepArgs(max_steps=8, ce_reduction="tokens", teacher_stream=teacher_stream, logits_chunk=chunk,
                    teacher_stream_sms=sms)
    trainer, shape = build_distill("cpu_tp2", "cpu", seed=3, args=args, tp=True)
    g = torch.Generator().manual_seed(9)
    with torch.no_grad():
        for layer in trainer.replaced.values():
            layer.gates.copy_(torch.randn(layer.num_candidates, generator=g))
    x, y = S.random_tokens(shape, "cpu", seed=5)
    log.clear()
    out = trainer.forward_backward(x, y)
    grads = {n: m.gates.grad.detach().clone() for n, m in trainer.replaced.items()}
    return float(out["loss"]), grads, list(log)


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    import cpu_kernels
    from voodoo_quant import parallel as P

    dist.init_process_group("gloo", rank=rank, world_size=world)
    _host_streams()
    from voodoo_quant.training import synthetic as S

    S.SHAPES["cpu_tp2"] = S.ModelShape(1, 512, 4, 2, 1024, 4096, False, head_dim=128,
                                       candidates=["Q4_K", "Q6_K", "Q8_0"], batch=2, seq=48, budget=0.45)
    log = []
    real = dist.all_reduce

    def logged(t, *a, group=None, **k):
        log.append("teacher" if group is not None and group is P.TP.teacher_group else "tp")
        return real(t, *a, group=group, **k)

    dist.all_reduce = logged
    undo = cpu_kernels.install()
    from voodoo_quant import _C

    reserves = []
    _C.set_gemm_sm_reserve = reserves.append  # (undo restores the library's setter)
    try:
        P.adopt_process_group(0)
        res = {}
        res["default0"] = _step(False, 0, log)
        for chunk in (0, 40):
            reserves.clear()
            res[f"stream{chunk}"] = _step(True, chunk, log, sms=16)
            res[f"reserves{chunk}"] = list(reserves)
        res["teacher_group_made"] = P.TP.teacher_group is not None
        torch.save(res, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.all_reduce = real
        undo()
        P.reset_tp()
        dist.destroy_process_group()


def test_teacher_stream_step_equals_the_default_step_tp2():
    world = 2
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_worker, args=(world, _free_port(), td), nprocs=world, join=True, start_method="spawn")
        rs = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(world)]
    for r in rs:
        assert r["teacher_group_made"]
        d = r["default0"]
        for chunk in (0, 40):
            s = r[f"stream{chunk}"]
            assert set(s[1]) == set(d[1])
            if chunk == 0:  # the same computation: bit for bit
                assert s[0] == d[0]
                assert all(torch.equal(s[1][n], d[1][n]) for n in d[1])
            else:  # head + loss per token chunk: the same sums in another order
                assert abs(s[0] - d[0]) <= 1e-5 * abs(d[0])
                assert all(float((s[1][n] - d[1][n]).norm()) <= 1e-4 * float(d[1][n].norm()) + 1e-12 for n in d[1])
            # default: every forward sum on the TP group; teacher stream: the
            # teacher's share (one per row-parallel layer and the embedding)
            # moves to its own communicator, the rest stays
            assert "teacher" not in d[2]
            # both forwards issued with 16 SMs left to collectives, then none
            assert r[f"reserves{chunk}"] == [16, 0], r[f"reserves{chunk}"]
            n_teacher = s[2].count("teacher")
            if chunk == 0:
                assert n_teacher >= 3 and s[2].count("tp") == len(d[2]) - n_teacher, (s[2], d[2])
            else:  # the chunked head's backward sums differ; the teacher's forward share does not
                assert n_teacher == r["stream0"][2].count("teacher"), (s[2], r["stream0"][2])
