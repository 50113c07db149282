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


def test_static_ptqr_embedding_routes_each_table_row_once(monkeypatch):
    """Static PTQR embedding: one candidate per table row (here row % K, a
    stand-in draw), every token's row decoded by its row's candidate; the
    backward is the mixture's straight-through Jacobian, as without PTQR."""
    import cpu_kernels
    from oracle import ggml_blocks
    from voodoo_quant import layers
    from voodoo_quant.quants import rtn

    types = ["Q4_K", "Q6_K", "Q8_0"]
    V, D, K = 64, 256, 3
    torch.manual_seed(4)
    w = torch.randn(V, D) * 0.02
    cand = {q: rtn.quantize(w, q) for q in types}
    ids = torch.randint(0, V, (2, 20))
    ids[1, :5] = ids[0, :5]  # repeated tokens
    g = torch.randn(2, 20, D)
    monkeypatch.setattr(layers, "_sample_token_routing", lambda probs, n: torch.arange(n) % K)
    undo = cpu_kernels.install()
    try:
        layers.set_static_shapes(True)
        emb = layers.MixedQuantEmbedding(V, D, types, w, candidate_bytes=cand, tensor_name="emb")
        with torch.no_grad():
            emb.gates.copy_(torch.tensor([0.3, -0.2, 0.5]))
        layers.set_ptqr(True)
        out = emb(ids)
        out.float().backward(g)
        routed_grad = emb.gates.grad.clone()
        emb.gates.grad = None
        layers.set_ptqr(False)
        emb(ids).float().backward(g)
        mixture_grad = emb.gates.grad.clone()
    finally:
        layers.set_ptqr(False)
        layers.set_static_shapes(False)
        undo()
    dec = [torch.from_numpy(ggml_blocks.dequantize(cand[q].numpy().reshape(-1), q, V, D)) for q in types]
    flat = ids.reshape(-1)
    expect = torch.stack([dec[int(i) % K][int(i)] for i in flat]).to(torch.bfloat16).reshape(2, 20, D)
    assert torch.equal(out.detach().to(torch.bfloat16), expect)
    assert torch.equal(routed_grad, mixture_grad)


class _FakeGraphState:
    capturing = False
    owner = None


class _FakeGraph:
    """Stands in for torch.cuda.CUDAGraph on the host: replay() runs the
    owner's forward_backward again while flagged as capturing (as a real
    replay runs what was recorded without the host code) and writes the
    results into the recorded output tensors in place."""

    def replay(self):
        t = _FakeGraphState.owner
        _FakeGraphState.capturing = True
        try:
            out = t.forward_backward(t._gx, t._gy)
        finally:
            _FakeGraphState.capturing = False
        for k, v in out.items():
            if torch.is_tensor(v):
                t._gout[k].copy_(v)


class _FakeCapture:
    def __init__(self, graph):
        self.graph = graph

    def __enter__(self):
        _FakeGraphState.capturing = True

    def __exit__(self, *exc):
        _FakeGraphState.capturing = False
        return False


def test_replayed_steps_equal_eager_steps(monkeypatch):
    """capture() / replay_step() control flow on the host, with a stand-in
    for the CUDA graph: each replay takes this step's temperature from the
    bank's device scalar (the recorded step never sets it), the new batch
    from the static inputs, and the eager update after it; three replayed
    steps give bit for bit the losses and gates of three eager steps."""
    import contextlib

    import cpu_kernels
    from voodoo_quant import layers
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training import trainer as TR

    class _Stream:
        def wait_stream(self, other):
            pass

    monkeypatch.setattr(torch.cuda, "Stream", _Stream)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: _Stream())
    monkeypatch.setattr(torch.cuda, "stream", lambda s: contextlib.nullcontext())
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: None)
    monkeypatch.setattr(torch.cuda, "CUDAGraph", _FakeGraph)
    monkeypatch.setattr(torch.cuda, "graph", _FakeCapture)
    monkeypatch.setattr(TR, "_capturing", lambda: _FakeGraphState.capturing)

    batches = [S.random_tokens(S.SHAPES["tiny"], "cpu", seed=20 + i) for i in range(3)]
    runs = {}
    undo = cpu_kernels.install()
    try:
        for mode in ("eager", "replay"):
            args = TR.StepArgs(max_steps=6, ce_reduction="tokens", static_shapes=True)
            trainer, _ = TR.build_distill("tiny", "cpu", seed=3, args=args)
            g = torch.Generator().manual_seed(9)
            with torch.no_grad():
                for layer in trainer.replaced.values():
                    layer.gates.copy_(torch.randn(layer.num_candidates, generator=g))
            if mode == "replay":
                _FakeGraphState.owner = trainer
                trainer.capture(*batches[0], warmup=2)
                step = trainer.replay_step
            else:
                step = trainer.step
            seq = []
            for x, y in batches:
                out = step(x, y)
                seq.append((float(out["loss"]), out["tau"],
                            [l.gates.detach().clone() for l in trainer.replaced.values()]))
            runs[mode] = seq
            trainer.release_graph()
    finally:
        undo()
        layers.set_static_shapes(False)
        _FakeGraphState.owner = None
    assert len({tau for _, tau, _ in runs["eager"]}) == 3  # the temperature moves every step
    for (le, te, ge), (lr_, tr_, gr) in zip(runs["eager"], runs["replay"]):
        assert le == lr_ and te == tr_
        assert all(torch.equal(a, b) for a, b in zip(ge, gr))


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
