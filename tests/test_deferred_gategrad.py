"""Overlap plumbing of the TP backward on CPU.

The gate-gradient GEMMs of an attention / MLP block can be deferred until the
all-reduce of the block's input gradient is in flight (the f operator's
backward), and a layer that sums its own input gradient can split dX into row
chunks whose all-reduces start one by one.  Both must leave every gradient
unchanged.  The CUDA kernels are replaced here by torch stand-ins (fp32
matmuls on dense candidate weights), so these tests check the autograd
wiring only: the gate bank's tap, the defer queue, the flush at the f
operator, the chunked all-reduce and the second communicator (gloo, world
size 1 and 2).  The kernels themselves are covered by the GPU tests.
"""

from __future__ import annotations

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp
import torch.nn as nn

TYPES = ["Q4_K", "Q8_0", "Q6_K"]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _install_fakes():
    """Swap the kernels the gated Linear calls for torch stand-ins; returns an undo."""
    from voodoo_quant import _C
    from voodoo_quant.layers import MixedQuantLinear

    def mix(self, probs):
        return (probs.float().view(-1, 1, 1) * torch.stack(self._test_w)).sum(0).to(torch.bfloat16)

    def linear_fwd(x, w, n_out=None, in_features=None, out=None):
        return (x.float() @ w.float().t()).to(torch.bfloat16)

    def linear_dx(dy, w, in_features, out=None):
        r = (dy.float() @ w.float()).to(torch.bfloat16)
        if out is None:
            return r
        out.copy_(r)
        return out

    def gategrad(dy, x, qtypes, qbytes, n_out, in_features, padded_cols, workspace=None, out=None):
        dw = dy.float().t() @ x.float()
        g = torch.stack([(dw * w).sum() for w in qbytes])
        if out is None:
            return g
        out.copy_(g)
        return out

    saved = []
    for obj, name, val in [(MixedQuantLinear, "_mix", mix),
                           (MixedQuantLinear, "_candidate_blocks", lambda self: self._test_w),
                           (MixedQuantLinear, "_gategrad_workspace", lambda self, dev: None),
                           (_C, "linear_fwd", linear_fwd), (_C, "linear_dx", linear_dx), (_C, "gategrad", gategrad),
                           (_C, "set_gategrad_sm_reserve", lambda n: None),
                           (_C, "set_gemm_sm_reserve", lambda n: None)]:
        saved.append((obj, name, obj.__dict__.get(name, None), name in obj.__dict__))
        setattr(obj, name, val)

    def undo():
        for obj, name, old, had in reversed(saved):
            if had:
                setattr(obj, name, old)
            else:
                delattr(obj, name)
    return undo


def _gated(in_f, out_f, w_full, name, spec=None):
    from voodoo_quant.layers import MixedQuantLinear
    from voodoo_quant.quants import rtn

    full = {q: rtn.quantize(w_full, q) for q in TYPES}
    if spec is None:
        w = w_full
    elif spec.row_offset is not None:
        w = w_full[spec.row_offset:spec.row_offset + spec.row_len]
    else:
        w = w_full[:, spec.col_offset:spec.col_offset + spec.col_len]
    m = MixedQuantLinear(in_f, out_f, TYPES, w, tensor_name=name, shard_spec=spec, candidate_bytes=full,
                         full_source_weight=None if spec is None else w_full)
    m._test_w = [w.float() * (1.0 + 0.15 * k) for k in range(len(TYPES))]
    with torch.no_grad():
        m.gates.copy_(torch.tensor([0.3, -0.2, 0.5]) * (1 + len(name) % 3))
    return m


class _Block(nn.Module):
    """q/k column-parallel, o row-parallel: y = o(tanh(q x) * k x)."""

    def __init__(self, q, k, o):
        super().__init__()
        self.q, self.k, self.o = q, k, o

    def forward(self, x):
        return self.o(torch.tanh(self.q(x).float()).to(torch.bfloat16) * self.k(x))


def _model(rank: int, world: int):
    from voodoo_quant.parallel import ShardSpec, block_aligned_split

    d, h = 256, 512
    g = torch.Generator().manual_seed(11)
    wq, wk = (torch.randn(h, d, generator=g) * 0.05 for _ in range(2))
    wo = torch.randn(d, h, generator=g) * 0.05
    if world == 1:
        return _Block(_gated(d, h, wq, "b.q"), _gated(d, h, wk, "b.k"), _gated(h, d, wo, "b.o"))
    off, n = block_aligned_split(h, world, rank)
    rs = ShardSpec(full_out=h, full_in=d, row_offset=off, row_len=n)
    cs = ShardSpec(full_out=d, full_in=h, col_offset=off, col_len=n)
    return _Block(_gated(d, n, wq, "b.q", rs), _gated(d, n, wk, "b.k", rs), _gated(n, d, wo, "b.o", cs))


def _run(rank: int, world: int, defer: bool):
    from voodoo_quant import parallel as P
    from voodoo_quant.layers import GateBank

    blk = _model(rank, world)
    root = nn.ModuleDict({"blk": blk})
    P._install_input_copy(blk)
    if defer:
        assert P.mark_deferred_gategrads(root) == 3
    bank = GateBank({"q": blk.q, "k": blk.k, "o": blk.o})
    assert bank.defer == defer
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 300, 256, generator=g).to(torch.bfloat16).requires_grad_(True)
    gy = torch.randn(2, 300, 256, generator=g)
    bank.probs()
    y = blk(x)
    loss = (y.float() * gy).sum() + 1e-6 * bank.effective_bytes()
    loss.backward()
    bank.release()
    from voodoo_quant import layers
    assert not layers.has_deferred_gategrads()
    return {"x": x.grad.float().clone(), **{n: getattr(blk, n).gates.grad.clone() for n in ("q", "k", "o")}}


def test_deferred_gategrads_single_process():
    undo = _install_fakes()
    try:
        a, b = _run(0, 1, defer=False), _run(0, 1, defer=True)
    finally:
        undo()
    for n in a:
        assert torch.equal(a[n], b[n]), n
    assert all(a[n].abs().sum() > 0 for n in ("q", "k", "o"))


def _chunk_run(rank: int, world: int, chunks: int):
    from voodoo_quant import layers
    from voodoo_quant.parallel import ShardSpec, block_aligned_split

    layers.INPUT_GRAD_CHUNKS = chunks
    try:
        d, h = 256, 512
        w = torch.randn(h, d, generator=torch.Generator().manual_seed(2)) * 0.05
        off, n = block_aligned_split(h, world, rank)
        m = _gated(d, n, w, "c.up", ShardSpec(full_out=h, full_in=d, row_offset=off, row_len=n))
        m.reduce_input_grad = True
        g = torch.Generator().manual_seed(9)
        x = torch.randn(600, d, generator=g).to(torch.bfloat16).requires_grad_(True)
        gy = torch.randn(600, h, generator=g)[:, off:off + n]
        (m(x).float() * gy).sum().backward()
        return {"x": x.grad.float().clone(), "g": m.gates.grad.clone()}
    finally:
        layers.INPUT_GRAD_CHUNKS = 1


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from voodoo_quant import parallel as P

    dist.init_process_group("gloo", rank=rank, world_size=world)
    undo = _install_fakes()
    try:
        P.adopt_process_group(0)
        res = {"plain": _run(rank, world, defer=False)}
        assert P.enable_input_grad_overlap(24) and P.TP.overlap_group is not None
        from voodoo_quant import layers

        flushes, orig = [], layers.flush_deferred_gategrads

        def spy(overlap_bytes=0):
            flushes.append((overlap_bytes, len(layers._DEFERRED)))
            return orig(overlap_bytes)

        layers.flush_deferred_gategrads = spy
        try:
            res["deferred"] = _run(rank, world, defer=True)
        finally:
            layers.flush_deferred_gategrads = orig
        # all three GEMMs ran beside the f operator's all-reduce of dX (600 x 256 bf16)
        assert flushes[0] == (600 * 256 * 2, 3) and all(n == 0 for _, n in flushes[1:]), flushes
        res["chunk1"] = _chunk_run(rank, world, 1)
        res["chunk3"] = _chunk_run(rank, world, 3)
        torch.save(res, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        undo()
        P.reset_tp()
        dist.destroy_process_group()


def test_deferred_and_chunked_input_grad_gloo_tp2():
    world = 2
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_worker, args=(world, _free_port(), td), nprocs=world, join=True, start_method="spawn")
        res = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(world)]
    undo = _install_fakes()
    try:
        ref = _run(0, 1, defer=False)
    finally:
        undo()
    for r in res:
        for n in ("x", "q", "k", "o"):
            assert torch.equal(r["plain"][n], r["deferred"][n]), n
        assert torch.equal(r["chunk1"]["x"], r["chunk3"]["x"])
        assert torch.equal(r["chunk1"]["g"], r["chunk3"]["g"])
    # the f operator makes every rank's input gradient the unsharded one
    assert torch.allclose(res[0]["deferred"]["x"], res[1]["deferred"]["x"])
    assert torch.allclose(res[0]["deferred"]["x"], ref["x"], rtol=0.05, atol=0.05)
    # gate gradients are rank-local partial sums (the trainer all-reduces them)
    for n in ("q", "k", "o"):
        assert torch.allclose(res[0]["deferred"][n] + res[1]["deferred"][n], ref[n], rtol=0.02, atol=1e-3), n


class _GroupedBlock(nn.Module):
    """q and k as one grouped gated projection: y = o(tanh(q x) * k x)."""

    def __init__(self, q, k, o, grouped: bool):
        super().__init__()
        self.q, self.k, self.o, self.grouped = q, k, o, grouped

    def forward(self, x):
        from voodoo_quant.layers import gated_linear_group

        if self.grouped:
            qk = gated_linear_group([self.q, self.k], x)
            q, k = qk.split([self.q.out_features, self.k.out_features], dim=-1)
        else:
            q, k = self.q(x), self.k(x)
        return self.o(torch.tanh(q.float()).to(torch.bfloat16) * k)


def test_grouped_gategrads_direct_and_deferred():
    """The gate gradients of a grouped q|k projection come from one grouped
    gate-gradient call -- written straight into the gate bank's gradient rows
    when deferred -- and equal those of the separate layers."""
    from voodoo_quant import _C, layers
    from voodoo_quant import parallel as P
    from voodoo_quant.layers import GateBank, groupable

    undo = _install_fakes()
    calls = []
    saved_mix, saved_grp = _C.__dict__.get("mix"), _C.__dict__.get("gategrad_grouped")

    def mix(qtypes, qbytes, probs, rows, padded, cols, out=None):
        w = (probs.float().view(-1, 1, 1) * torch.stack(qbytes)).sum(0).to(torch.bfloat16)
        if out is None:
            return w
        out[:, :cols].copy_(w[:, :cols])
        return out

    def gategrad_grouped(dy, x, qtypes, qbytes_per_layer, rows, in_features, padded_cols, workspace=None, out=None):
        calls.append(tuple(rows))
        g, a = [], 0
        for n, qb in zip(rows, qbytes_per_layer):
            g.append(_C.gategrad(dy[:, a:a + n], x, qtypes, qb, n, in_features, padded_cols))
            a += n
        g = torch.stack(g)
        if out is None:
            return g
        out.copy_(g)
        return out

    _C.mix, _C.gategrad_grouped = mix, gategrad_grouped
    _C.gategrad_grouped_workspace_bytes = lambda n, k, g, c: 4
    try:
        d, h = 256, 512
        gen = torch.Generator().manual_seed(11)
        wq, wk = (torch.randn(h, d, generator=gen) * 0.05 for _ in range(2))
        wo = torch.randn(d, h, generator=gen) * 0.05
        res = {}
        for grouped, defer in ((False, False), (True, False), (True, True)):
            blk = _GroupedBlock(_gated(d, h, wq, "b.q"), _gated(d, h, wk, "b.k"), _gated(h, d, wo, "b.o"), grouped)
            if grouped:
                assert groupable([blk.q, blk.k])
            root = nn.ModuleDict({"blk": blk})
            P._install_input_copy(blk)
            if defer:
                assert P.mark_deferred_gategrads(root) == 3
            bank = GateBank({"q": blk.q, "k": blk.k, "o": blk.o})
            g = torch.Generator().manual_seed(5)
            x = torch.randn(2, 300, d, generator=g).to(torch.bfloat16).requires_grad_(True)
            gy = torch.randn(2, 300, d, generator=g)
            bank.probs()
            del calls[:]
            loss = (blk(x).float() * gy).sum()
            loss.backward()
            bank.release()
            assert not layers.has_deferred_gategrads()
            assert calls == ([(h, h)] if grouped else []), calls
            res[(grouped, defer)] = {"x": x.grad.float().clone(),
                                     **{n: getattr(blk, n).gates.grad.clone() for n in ("q", "k", "o")}}
    finally:
        for name, old in (("mix", saved_mix), ("gategrad_grouped", saved_grp)):
            setattr(_C, name, old)
        del _C.gategrad_grouped_workspace_bytes
        undo()
    base = res[(False, False)]
    for key in ((True, False), (True, True)):
        # dX: one GEMM over both layers' columns instead of two bf16 dX added
        assert float((res[key]["x"] - base["x"]).norm()) <= 1e-2 * float(base["x"].norm()), key
        for n in ("q", "k", "o"):
            assert torch.allclose(res[key][n], base[n], rtol=1e-5, atol=1e-6), (key, n)
    for n in ("q", "k", "o"):
        assert torch.equal(res[(True, False)][n], res[(True, True)][n]), n
