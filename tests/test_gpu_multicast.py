"""Row-parallel GEMM with the all-reduce fused into its epilogue
(vq_linear_fwd_mcred through parallel.MulticastReducer) against the same
GEMM followed by an NCCL all-reduce, on 2 GPUs (skipped with fewer).

Tolerance: 1e-2 relative (L2): both sum bf16 partial outputs; the switch and
the NCCL ring add them in different orders.
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
    import sys
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    from voodoo_quant import _C, parallel

    res = {}
    try:
        parallel.adopt_process_group(rank)
        red = parallel.enable_multicast_reduce(True)
        res["available"] = red is not None
        if red is not None:
            errs = []
            for i, (T, N, K) in enumerate([(512, 1024, 768), (2048, 4096, 512), (300, 1024, 256), (2048, 4096, 512)]):
                g = torch.Generator(device="cpu").manual_seed(100 * i + rank)
                x = torch.randn(T, K, generator=g).to(dev, torch.bfloat16)
                w = (torch.randn(N, K, generator=g) * 0.05).to(dev, torch.bfloat16)
                y = red.linear(x, w, N, K)
                ref = _C.linear_fwd(x, w, N, K).float()
                dist.all_reduce(ref)
                errs.append(float((y.float() - ref).norm() / ref.norm()))
            res["errs"] = errs
            res["dev_err"] = _C.device_error()
        parallel.enable_multicast_reduce(False)
        torch.save(res, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        parallel.reset_tp()
        dist.destroy_process_group()


def test_fused_row_parallel_allreduce_matches_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    port = _free_port()
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_worker, args=(2, port, td), nprocs=2, join=True, start_method="spawn")
        rs = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(2)]
    if not rs[0]["available"]:
        pytest.skip("NVLink multicast not available")
    for r in rs:
        assert r["dev_err"] == 0
        assert max(r["errs"]) < 1e-2, r["errs"]
