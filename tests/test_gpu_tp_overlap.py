"""TP-2 distillation step with the input-gradient all-reduces overlapped
(gate-gradient GEMMs deferred beside them on a second communicator; then
also the head's dX all-reduced in two row chunks) against the same step
without overlap, and the sequence-parallel step (token-shard residual
stream, all-gather / reduce-scatter around every block) with and without
the overlap, and the step whose TP-1 teacher runs interleaved with the
student's forward all-reduces against the same teacher run after the
student, on 2 GPUs (skipped with fewer).

The overlap only reorders launches and leaves SMs free; the gate-gradient
GEMM's stream-K split depends on how many SMs it gets, so its fp32 partial
sums may be added in another order.  Tolerance: loss 1e-5 relative, gate
gradients 1e-3 relative per tensor (L2).  Sequence parallelism sums the
row-parallel outputs by reduce-scatter instead of all-reduce (another order
of the bf16 partial sums): loss 2e-3 relative, gate gradients per tensor
within 3e-2 relative with cosine >= 0.999.
"""

from __future__ import annotations

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    from voodoo_quant import _C, layers, parallel
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    # the smallest Llama shape whose TP-2 shards keep every input dimension 256-aligned
    S.SHAPES["tp2_test"] = S.ModelShape(2, 512, 4, 2, 1024, 4096, False, head_dim=128,
                                        candidates=["Q4_K", "Q6_K", "Q8_0"], batch=2, seq=256)
    res = {}
    try:
        parallel.adopt_process_group(rank)
        for sms, chunks, sp, extra in ((0, 1, False, None), (24, 1, False, None), (24, 2, False, None),
                                       (0, 1, True, None), (24, 1, True, None), (24, 1, False, "tt1"),
                                       (24, 1, False, "joint")):
            layers.INPUT_GRAD_CHUNKS = chunks  # the head sums its own input gradient in row chunks
            kw = {} if extra is None else {"teacher_tp": 1, "joint_teacher": extra == "joint"}
            trainer, shape = build_distill("tp2_test", dev, seed=0, tp=True, overlap_sms=sms,
                                           args=StepArgs(sequence_parallel=sp, **kw))
            joint = trainer._joint_ok()
            deferred = sum(bool(m.__dict__.get("_defer_gategrad", False)) for m in trainer.replaced.values())
            x, y = S.random_tokens(shape, dev, seed=1)
            out = trainer.forward_backward(x, y)
            torch.cuda.synchronize()
            res[extra or (sms, chunks, sp)] = {"loss": float(out["loss"]), "deferred": deferred, "joint": joint,
                        "grads": {n: m.gates.grad.detach().cpu().clone() for n, m in trainer.replaced.items()},
                        "left": layers.has_deferred_gategrads()}
            del trainer
        layers.INPUT_GRAD_CHUNKS = 1
        res["dev_err"] = _C.device_error()
        torch.save(res, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        parallel.reset_tp()
        dist.destroy_process_group()


def test_overlapped_input_grad_allreduce_matches_plain_step():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_worker, args=(2, _free_port(), td), nprocs=2, join=True, start_method="spawn")
        rs = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(2)]
    for r in rs:
        assert r["dev_err"] == 0
        a = r[(0, 1, False)]
        assert a["deferred"] == 0
        for key in ((24, 1, False), (24, 2, False), (24, 1, True)):
            b = r[key]
            base = r[(0, 1, key[2])]
            assert b["deferred"] > 0 and not b["left"]
            assert abs(base["loss"] - b["loss"]) <= 1e-5 * abs(base["loss"])
            for n, g in base["grads"].items():
                h = b["grads"][n]
                assert float((g - h).norm()) <= 1e-3 * float(g.norm()) + 1e-12, (key, n)
        # the teacher (TP-1, each rank's batch slice) interleaved with the
        # student's forward all-reduces: the same step
        tt1, joint = r["tt1"], r["joint"]
        assert joint["joint"] and not tt1["joint"]
        assert abs(tt1["loss"] - joint["loss"]) <= 1e-5 * abs(tt1["loss"])
        for n, g in tt1["grads"].items():
            assert float((g - joint["grads"][n]).norm()) <= 1e-3 * float(g.norm()) + 1e-12, n
        sp = r[(0, 1, True)]
        assert abs(sp["loss"] - a["loss"]) <= 2e-3 * abs(a["loss"])
        for n, g in a["grads"].items():
            h = sp["grads"][n].double()
            gd = g.double()
            assert float((h - gd).norm()) <= 3e-2 * float(gd.norm()) + 1e-12, n
            assert float(h @ gd) >= 0.999 * float(h.norm() * gd.norm()), n
