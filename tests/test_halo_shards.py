"""Halo shards: row-parallel inputs whose rank-local width is whole attention
heads but not whole 256-weight blocks (the 32B shape's o_proj at TP-8: 5
heads x 128 = 640 columns per rank).  The rank stores the packed blocks that
cover its columns and multiplies through a column window of its mixed
weight; its gate gradient sees zero inputs outside the window.

CPU only: packed-block slicing against packing the covering columns, the
gated row-parallel layer and the Q8_0 teacher layer against their unsharded
forms (kernels replaced by the torch stand-ins of tests/cpu_kernels.py), the
per-role candidate menus, and a whole TP-2 distillation step over gloo with a
halo o_proj against one process.

Tolerances: block bytes exact; summed partial outputs 1e-2 relative (each
rank's output is rounded to bf16 before the sum); input gradients exact
(each rank's columns are computed alone); gate gradients 1e-5 relative
(fp32 dots of the same bf16 products, summed in another order); the TP-2
step as tests/test_trainer_cpu_fakes.py (loss 2e-2, gate-gradient cosine
>= 0.999).
"""

from __future__ import annotations

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

HALO_TYPES = ["Q2_K", "Q3_K", "Q4_K", "IQ4_XS", "Q6_K", "Q8_0"]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("fmt", HALO_TYPES)
def test_halo_slice_equals_packing_the_covering_columns(fmt):
    from voodoo_quant.parallel import ShardSpec
    from voodoo_quant.quants import rtn

    torch.manual_seed(0)
    w = torch.randn(24, 1280) * 0.02
    full = rtn.quantize(w, fmt)
    # 1280 = 10 heads x 128 over two ranks: 640 columns each, 2.5 blocks
    for r, (units, off) in enumerate([((0, 3), 0), ((2, 5), 128)]):
        spec = ShardSpec(full_out=24, full_in=1280, col_offset=640 * r, col_len=640, halo=True)
        assert spec.col_units() == units and spec.in_col_offset == off
        assert spec.local_padded_in(1280, [fmt]) == 768
        assert torch.equal(spec.local_block_weight(w), w[:, units[0] * 256:units[1] * 256])
        assert torch.equal(spec.slice_qbytes(full, fmt, 1280).reshape(-1),
                           rtn.quantize(w[:, units[0] * 256:units[1] * 256], fmt).reshape(-1))
        # without the halo flag the reference's refusal stands
        plain = ShardSpec(full_out=24, full_in=1280, col_offset=640 * r, col_len=640)
        with pytest.raises(ValueError, match="aligned"):
            plain.slice_qbytes(full, fmt, 1280)

    # the last rank's blocks reach into the zero padding of a 640-wide tensor
    w2 = torch.randn(8, 640) * 0.02
    padded = torch.nn.functional.pad(w2, (0, 128))
    spec = ShardSpec(full_out=8, full_in=640, col_offset=320, col_len=320, halo=True)
    assert spec.col_units() == (1, 3) and spec.in_col_offset == 64
    assert torch.equal(spec.local_block_weight(w2), padded[:, 256:768])
    assert torch.equal(spec.slice_qbytes(rtn.quantize(padded, fmt), fmt, 768).reshape(-1),
                       rtn.quantize(padded[:, 256:768], fmt).reshape(-1))


@pytest.mark.parametrize("fmt", HALO_TYPES)
def test_packing_the_rank_part_equals_slicing_the_full_packing(fmt):
    """The synthetic candidate provider packs only a rank's part under TP
    (``ShardSpec.local_block_weight``); for every kind of shard -- rows, a
    row index, block-aligned columns, halo columns, vocabulary rows of a
    tensor whose width is not a multiple of 256 -- that equals the rank's
    slice of the packed full tensor."""
    from voodoo_quant.parallel import ShardSpec
    from voodoo_quant.quants import rtn

    torch.manual_seed(3)
    w = torch.randn(40, 1280) * 0.02
    w_odd = torch.randn(24, 640) * 0.02  # padded to 768 for packing
    specs = [
        (w, ShardSpec(full_out=40, full_in=1280, row_offset=8, row_len=20)),
        (w, ShardSpec(full_out=40, full_in=1280, row_index=torch.tensor([3, 1, 30, 7, 22]))),
        (w, ShardSpec(full_out=40, full_in=1280, col_offset=512, col_len=768)),
        (w, ShardSpec(full_out=40, full_in=1280, col_offset=640, col_len=640, halo=True)),
        (w_odd, ShardSpec(full_out=24, full_in=640, row_offset=12, row_len=12, vocab_start=12)),
        (w_odd, ShardSpec(full_out=24, full_in=640, col_offset=320, col_len=320, halo=True)),
    ]
    for full_w, spec in specs:
        padded = torch.nn.functional.pad(full_w, (0, -full_w.shape[1] % 256))
        whole = rtn.quantize(padded, fmt)
        local = rtn.quantize(spec.local_block_weight(full_w), fmt)
        assert torch.equal(local.reshape(-1), spec.slice_qbytes(whole, fmt, padded.shape[1]).reshape(-1)), spec


def test_32b_tp8_o_proj_geometry():
    """Every TP-8 rank of the 32B o_proj (5120 = 40 heads x 128) stores three
    blocks, starts at column 0 or 128 inside them, and the ranks' exact
    columns tile the row once."""
    from voodoo_quant.parallel import ShardSpec

    seen = torch.zeros(5120, dtype=torch.int32)
    for r in range(8):
        spec = ShardSpec(full_out=5120, full_in=5120, col_offset=640 * r, col_len=640, halo=True)
        u0, u1 = spec.col_units()
        assert u1 - u0 == 3 and spec.local_padded_in(5120, ["Q4_K"]) == 768
        assert spec.in_col_offset == (0 if r % 2 == 0 else 128)
        assert spec.in_col_offset % 8 == 0  # 16-byte aligned bf16 column window
        lo = u0 * 256 + spec.in_col_offset
        seen[lo:lo + 640] += 1
    assert bool((seen == 1).all())


def _layer(types, w, bytes_full, probs_gates, spec=None):
    from voodoo_quant.layers import MixedQuantLinear

    out_f, in_f = w.shape
    if spec is not None:
        in_f = spec.local_in
    layer = MixedQuantLinear(in_f, out_f, types, spec.slice_weight(w) if spec is not None else w,
                             shard_spec=spec, full_source_weight=w if spec is not None else None,
                             candidate_bytes=bytes_full, tensor_name="halo.o_proj")
    with torch.no_grad():
        layer.gates.copy_(probs_gates)
    return layer


@pytest.mark.parametrize("width", [640, 320])  # 2 ranks (offsets 0, 128) / 4 ranks (0, 64, 128, 192)
def test_halo_row_parallel_layer_sums_to_the_full_layer(width):
    import cpu_kernels
    from voodoo_quant.parallel import ShardSpec
    from voodoo_quant.quants import rtn

    types = ["Q3_K", "IQ4_XS", "Q6_K", "Q8_0"]
    torch.manual_seed(1)
    out_f, in_f, T = 40, 1280, 24
    w = torch.randn(out_f, in_f) * 0.02
    cand = {q: rtn.quantize(w, q) for q in types}
    gates = torch.randn(len(types))
    x = torch.randn(T, in_f).to(torch.bfloat16)
    dy = torch.randn(T, out_f).to(torch.bfloat16)
    undo = cpu_kernels.install()
    try:
        full = _layer(types, w, cand, gates)
        xf = x.clone().requires_grad_(True)
        yf = full(xf)
        yf.backward(dy)
        y_sum = torch.zeros(T, out_f)
        g_sum = torch.zeros(len(types))
        for r in range(in_f // width):
            c0, c1 = width * r, width * (r + 1)
            spec = ShardSpec(full_out=out_f, full_in=in_f, col_offset=c0, col_len=width, halo=True)
            part = _layer(types, w, cand, gates, spec)
            assert part.in_col_offset == c0 % 256
            assert part.padded_in_features == ((c1 + 255) // 256 - c0 // 256) * 256
            assert part._w_0.shape == (out_f, width)
            assert torch.equal(part._w_2, full._w_2[:, c0:c1])
            assert torch.equal(part.get_mixed_weight(), full.get_mixed_weight()[:, c0:c1])
            xr = x[:, c0:c1].clone().requires_grad_(True)
            yr = part(xr)
            yr.backward(dy)
            y_sum += yr.detach().float()
            g_sum += part.gates.grad
            assert torch.equal(xr.grad, xf.grad[:, c0:c1]), r
    finally:
        undo()
    yf = yf.detach().float()
    assert float((y_sum - yf).norm()) <= 1e-2 * float(yf.norm())
    assert float((g_sum - full.gates.grad).norm()) <= 1e-5 * float(full.gates.grad.norm())


def test_q8_teacher_halo_layer_uses_the_covering_blocks():
    import cpu_kernels
    from voodoo_quant.parallel import ShardSpec
    from voodoo_quant.quants import rtn
    from voodoo_quant.training.q8_teacher import Q8Linear

    torch.manual_seed(2)
    w = torch.randn(16, 1280) * 0.02
    full = Q8Linear(rtn.quantize(w, "Q8_0"), 16, 1280)
    undo = cpu_kernels.install()
    try:
        wf = full.weight_bf16()
        for r in range(2):
            spec = ShardSpec(full_out=16, full_in=1280, col_offset=640 * r, col_len=640, halo=True)
            part = Q8Linear(rtn.quantize(spec.local_block_weight(w), "Q8_0"), 16, 640,
                            padded_in=spec.local_padded_in(1280, ["Q8_0"]), in_col_offset=spec.in_col_offset)
            assert torch.equal(part.weight_bf16(), wf[:, 640 * r:640 * (r + 1)])
    finally:
        undo()
    with pytest.raises(ValueError):
        Q8Linear(rtn.quantize(w[:, :768], "Q8_0"), 16, 640, padded_in=768, in_col_offset=200)


def _shapes():
    from voodoo_quant.training import synthetic as S

    # the 32B shape's TP-8 o_proj geometry at TP-2: 10 heads x 128 = 1280,
    # 640 columns per rank; ffn 1792 = 7 blocks splits 4 / 3; per-role menus
    # and per-row log-normal weight scales as in the 32B shape
    S.SHAPES["cpu_halo"] = S.ModelShape(
        1, 1280, 10, 2, 1792, 4096, False, head_dim=128, candidates=["IQ4_XS", "Q3_K", "Q4_K", "Q8_0", "Q2_K"],
        attention_candidates=["Q4_K", "IQ4_XS", "Q8_0"], non_attention_candidates=["IQ4_XS", "Q3_K", "Q4_K",
                                                                                    "Q8_0", "Q2_K"],
        batch=2, seq=24, budget=0.30, row_scale_sigma=0.5)


def _step(tp: bool, overlap_sms: int = 0):
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    trainer, shape = build_distill("cpu_halo", "cpu", seed=3, args=StepArgs(max_steps=4, ce_reduction="tokens"),
                                   tp=tp, overlap_sms=overlap_sms)
    if overlap_sms:  # the halo o_proj's gate-gradient GEMM is deferred beside the input-gradient all-reduce
        assert trainer.replaced["model.layers.0.self_attn.o_proj"].__dict__.get("_defer_gategrad", False)
    x, y = S.random_tokens(shape, "cpu", seed=5)
    r = trainer.forward_backward(x, y)
    grads = {n: m.gates.grad.detach().clone() for n, m in trainer.replaced.items()}
    menus = {n: list(m.candidate_types) for n, m in trainer.replaced.items()}
    offsets = {n: m.in_col_offset for n, m in trainer.replaced.items()}
    return float(r["loss"]), grads, menus, offsets


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
        # plain, and with the gate-gradient GEMMs deferred beside the input-gradient
        # all-reduces (the benchmark's TP default)
        torch.save({"plain": _step(True), "deferred": _step(True, overlap_sms=24)},
                   os.path.join(outdir, f"r{rank}.pt"))
    finally:
        undo()
        P.reset_tp()
        dist.destroy_process_group()


def _cos(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double().flatten(), b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm() + 1e-300))


def test_tp2_step_with_halo_o_proj_matches_one_process():
    pytest.importorskip("transformers")
    import cpu_kernels

    world = 2
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_worker, args=(world, _free_port(), td), nprocs=world, join=True, start_method="spawn")
        rs = [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(world)]
    _shapes()
    undo = cpu_kernels.install()
    try:
        ref = _step(False)
    finally:
        undo()
    o_proj = "model.layers.0.self_attn.o_proj"
    assert ref[2][o_proj] == ["Q4_K", "IQ4_XS", "Q8_0"]
    assert ref[2]["model.layers.0.mlp.down_proj"] == ["IQ4_XS", "Q3_K", "Q4_K", "Q8_0", "Q2_K"]
    assert [r["plain"][3][o_proj] for r in rs] == [0, 128]
    for rr in rs:
        r = rr["plain"]
        assert r[2] == ref[2]
        assert abs(r[0] - ref[0]) <= 2e-2 * abs(ref[0])
        for n, g in ref[1].items():
            assert _cos(r[1][n], g) > 0.999, n
            assert float((r[1][n] - g).norm()) <= 2e-2 * float(g.norm()) + 1e-9, n
        # deferring the GEMMs changes when they run, not a value
        d = rr["deferred"]
        assert d[0] == r[0]
        assert all(torch.equal(d[1][n], r[1][n]) for n in r[1])
    for n in ref[1]:
        assert torch.equal(rs[0]["plain"][1][n], rs[1]["plain"][1][n]), n
