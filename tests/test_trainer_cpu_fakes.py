"""The distillation step's host logic on CPU, with the CUDA kernels replaced
by torch stand-ins (tests/cpu_kernels.py): the gate bank, the head + loss
per token chunk, and tensor parallelism over gloo with and without the
deferred gate-gradient overlap.  The stand-ins are consistent with each
other, so these tests check the wiring, not the kernels (the GPU tests do).

Tolerances: chunked vs full logits 1e-5 relative (same arithmetic, summed
per chunk); TP-2 vs one process 2e-2 relative (bf16 partial sums added
across ranks) with gate-gradient cosine >= 0.999; the overlap on or off
exactly equal.
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

    # the smallest Llama shape whose TP-2 shards keep every input dimension 256-aligned
    S.SHAPES["cpu_tp2"] = S.ModelShape(1, 512, 4, 2, 1024, 4096, False, head_dim=128,
                                       candidates=["Q4_K", "Q6_K", "Q8_0"], batch=2, seq=48, budget=0.45)
    S.SHAPES["cpu_tied"] = S.ModelShape(2, 256, 4, 4, 768, 4096, True, candidates=["Q4_K", "Q5_K", "Q8_0"],
                                        batch=2, seq=48, budget=0.45)


def _step(name: str, tp: bool, overlap_sms: int, chunk: int, sp: bool = False, **step_args):
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    args = StepArgs(max_steps=4, ce_reduction="tokens", logits_chunk=chunk, sequence_parallel=sp, **step_args)
    trainer, shape = build_distill(name, "cpu", seed=3, args=args, tp=tp, overlap_sms=overlap_sms)
    x, y = S.random_tokens(shape, "cpu", seed=5)
    r = trainer.forward_backward(x, y)
    grads = {n: m.gates.grad.detach().clone() for n, m in trainer.replaced.items()}
    deferred = sum(bool(m.__dict__.get("_defer_gategrad", False)) for m in trainer.replaced.values())
    from voodoo_quant.parallel import sp_enabled
    on = sp_enabled() and hasattr(trainer.student.model, "_vq_sp_orig_forward")
    return float(r["loss"]), grads, deferred, on, trainer._joint_ok()


def _cos(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double().flatten(), b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-300))


@pytest.mark.parametrize("name", ["cpu_tp2", "cpu_tied"])
def test_chunked_head_matches_full_logits(name):
    import cpu_kernels

    _shapes()
    undo = cpu_kernels.install()
    try:
        full = _step(name, False, 0, 0)
        chunked = _step(name, False, 0, 40)  # 96 tokens: chunks of 40, 40 and 16
    finally:
        undo()
    assert abs(full[0] - chunked[0]) <= 1e-5 * abs(full[0])
    assert set(full[1]) == set(chunked[1])
    for n, g in full[1].items():
        assert float((g - chunked[1][n]).norm()) <= 1e-5 * float(g.norm()) + 1e-9, n


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    import cpu_kernels
    from voodoo_quant import parallel as P

    dist.init_process_group("gloo", rank=rank, world_size=world)
    _shapes()
    undo = cpu_kernels.install()
    try:
        P.adopt_process_group(0)
        res = {"plain": _step("cpu_tp2", True, 0, 0)}
        res["overlap"] = _step("cpu_tp2", True, 24, 0)
        res["overlap_chunked"] = _step("cpu_tp2", True, 24, 40)
        res["sp"] = _step("cpu_tp2", True, 0, 0, sp=True)
        res["sp_overlap"] = _step("cpu_tp2", True, 24, 0, sp=True)
        res["sp_chunked"] = _step("cpu_tp2", True, 24, 40, sp=True)
        res["tt1"] = _step("cpu_tp2", True, 24, 0, teacher_tp=1)
        res["joint"] = _step("cpu_tp2", True, 24, 0, teacher_tp=1, joint_teacher=True)
        torch.save(res, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        undo()
        P.reset_tp()
        dist.destroy_process_group()


def test_tp2_step_matches_one_process_with_and_without_overlap():
    import cpu_kernels

    world = 2
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_worker, args=(world, _free_port(), td), nprocs=world, join=True, start_method="spawn")
        rs = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(world)]
    _shapes()
    undo = cpu_kernels.install()
    try:
        ref = _step("cpu_tp2", False, 0, 0)
    finally:
        undo()
    for r in rs:
        plain, ov, ovc = r["plain"], r["overlap"], r["overlap_chunked"]
        assert plain[2] == 0 and ov[2] > 0 and ovc[2] > 0
        assert ov[0] == plain[0]
        assert abs(ovc[0] - plain[0]) <= 1e-5 * abs(plain[0])
        assert abs(plain[0] - ref[0]) <= 2e-2 * abs(ref[0])
        for n, g in ref[1].items():
            assert torch.equal(plain[1][n], ov[1][n]), n
            assert float((ovc[1][n] - ov[1][n]).norm()) <= 1e-4 * float(ov[1][n].norm()) + 1e-9, n
            assert _cos(plain[1][n], g) > 0.999, n
            assert float((plain[1][n] - g).norm()) <= 2e-2 * float(g.norm()) + 1e-9, n
    # sequence parallelism: the same step (token-shard residual stream,
    # all-gather / reduce-scatter around each block), with and without the
    # deferred gate-gradient overlap and with the chunked head
    for r in rs:
        sp, spo, spc = r["sp"], r["sp_overlap"], r["sp_chunked"]
        assert sp[3] and spo[3] and spc[3] and not r["plain"][3]
        assert sp[2] == 0 and spo[2] > 0
        assert abs(sp[0] - ref[0]) <= 2e-2 * abs(ref[0]) and abs(spo[0] - sp[0]) <= 1e-6 * abs(sp[0])
        assert abs(spc[0] - sp[0]) <= 1e-5 * abs(sp[0])
        for n, g in ref[1].items():
            assert _cos(sp[1][n], g) > 0.999, n
            assert float((sp[1][n] - g).norm()) <= 2e-2 * float(g.norm()) + 1e-9, n
            assert float((spo[1][n] - sp[1][n]).norm()) <= 1e-5 * float(sp[1][n].norm()) + 1e-9, n
            assert float((spc[1][n] - sp[1][n]).norm()) <= 1e-4 * float(sp[1][n].norm()) + 1e-9, n
    # the teacher's layers interleaved with the student's forward all-reduces
    # (teacher at TP-1 on each rank's batch slice): the same step exactly
    for r in rs:
        tt1, joint = r["tt1"], r["joint"]
        assert joint[4] and not tt1[4]
        assert joint[0] == tt1[0]
        for n in ref[1]:
            assert torch.equal(joint[1][n], tt1[1][n]), n
    # both ranks hold the same (all-reduced) gate gradients
    for n in ref[1]:
        assert torch.equal(rs[0]["plain"][1][n], rs[1]["plain"][1][n]), n
        assert torch.equal(rs[0]["sp"][1][n], rs[1]["sp"][1][n]), n


def test_ptqr_step_with_concentrated_gates_equals_the_mixture():
    """PTQR routes each token to one sampled candidate; with every gate
    distribution concentrated on one candidate (low temperature, large gate
    margin) the routed step and the mixture step give the same loss."""
    import cpu_kernels
    from voodoo_quant.layers import set_ptqr
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    _shapes()
    undo = cpu_kernels.install()
    out = {}
    try:
        for ptqr in (False, True):
            args = StepArgs(max_steps=4, ce_reduction="tokens", ptqr=ptqr, temp_start=0.05, temp_end=0.05)
            trainer, shape = build_distill("cpu_tied", "cpu", seed=3, args=args)
            for m in trainer.replaced.values():
                with torch.no_grad():
                    m.gates.zero_()
                    m.gates[-1] = 5.0  # the last candidate wins with probability ~1 at tau = 0.05
            x, y = S.random_tokens(shape, "cpu", seed=5)
            r = trainer.forward_backward(x, y)
            out[ptqr] = float(r["loss"])
            assert all(torch.isfinite(m.gates.grad).all() for m in trainer.replaced.values())
    finally:
        set_ptqr(False)
        undo()
    assert abs(out[True] - out[False]) <= 1e-4 * abs(out[False]), out
