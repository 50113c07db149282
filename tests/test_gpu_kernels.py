"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle.

Bit-exact: block decoding.  Within tolerance (bf16 inputs, fp32 accumulate,
compared with float64/float32 references): mixture, GEMMs, gate gradient,
fused loss.  Sizes are chosen so the oracle finishes in seconds; full-size
behaviour is covered by size-independent properties at the end.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cosine, rel_err, same_bits
from oracle import ggml_blocks, loss as oloss, mixgemm

pytestmark = pytest.mark.gpu

FORMATS = list(ggml_blocks.FORMATS)
TOL_GEMM = 1e-2        # relative (Frobenius) error, bf16 operands vs fp64 reference
TOL_COS = 0.999        # gate-gradient cosine, per tensor


@pytest.fixture(scope="module")
def dq(golden_dir):
    return np.load(golden_dir / "dequant_golden.npz")


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("tag", ["regular", "edge"])
def test_dequant_golden_bit_exact(cuda, dq, fmt, tag):
    from voodoo_quant import _C

    raw = dq[f"{fmt}/{tag}/bytes"]
    exp = dq[f"{fmt}/{tag}/expected"]
    got = _C.dequant(torch.from_numpy(raw).to(cuda), fmt, exp.shape[0], exp.shape[1])
    assert same_bits(got.cpu().numpy(), exp)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("rows,cols", [(1, 256), (3, 768), (37, 4096), (129, 2304)])
def test_dequant_random_blocks_bit_exact(cuda, fmt, rows, cols):
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn

    torch.manual_seed(rows * 7 + cols)
    w = torch.randn(rows, cols) * 0.03
    qb = rtn.quantize(w, fmt)
    got = _C.dequant(qb.to(cuda), fmt, rows, cols).cpu().numpy()
    assert same_bits(got, ggml_blocks.dequantize(qb.numpy(), fmt, rows, cols))


@pytest.mark.parametrize("cols", [32, 96, 480])
def test_dequant_q8_0_partial_units(cuda, cols):
    """Q8_0 rows need only be a multiple of 32 weights for the plain decoder."""
    from voodoo_quant import _C

    rng = np.random.default_rng(cols)
    rows = 5
    raw = rng.integers(0, 256, size=(rows * cols // 32, 34), dtype=np.uint8)
    raw[:, 0:2] = (rng.uniform(-0.01, 0.01, raw.shape[0]).astype(np.float16)).view(np.uint8).reshape(-1, 2)
    got = _C.dequant(torch.from_numpy(raw).to(cuda), "Q8_0", rows, cols).cpu().numpy()
    assert same_bits(got, ggml_blocks.dequantize(raw, "Q8_0", rows, cols))


def test_dequant_errors(cuda):
    from voodoo_quant import _C

    with pytest.raises(ValueError):
        _C.dequant(torch.zeros(144, dtype=torch.uint8, device=cuda), "Q4_K", 1, 100)
    with pytest.raises(ValueError):
        _C.dequant(torch.zeros(100, dtype=torch.uint8, device=cuda), "Q4_K", 1, 256)
    with pytest.raises(ValueError):
        _C.dequant(torch.zeros(66, dtype=torch.uint8, device=cuda), "IQ2_XXS", 1, 256)
    assert _C.device_error() == 0


def _cands(types, rows, padded, seed=0, scale=0.02):
    from voodoo_quant.quants import rtn

    g = torch.Generator().manual_seed(seed)
    w = torch.randn(rows, padded, generator=g) * scale
    return w, {q: rtn.quantize(w, q) for q in types}


@pytest.mark.parametrize("types,rows,cols", [
    (["Q4_K", "Q5_K", "Q6_K", "Q8_0"], 64, 512),
    (["Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 33, 1000),
    (["IQ4_XS", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "Q2_K"], 17, 768),
    (["Q8_0"], 8, 256),
])
def test_mix_matches_oracle(cuda, types, rows, cols):
    from voodoo_quant import _C

    padded = (cols + 255) // 256 * 256
    _, cb = _cands(types, rows, padded, seed=rows)
    probs = torch.softmax(torch.randn(len(types)), 0)
    w = _C.mix(types, [cb[q].to(cuda) for q in types], probs.to(cuda), rows, padded, cols)
    ld = (cols + 7) // 8 * 8
    assert w.shape == (rows, ld) and w.dtype == torch.bfloat16
    cands = mixgemm.decode_candidates([cb[q].numpy() for q in types], types, rows, padded, cols)
    ref = mixgemm.mixed_weight(cands, probs.numpy(), fp64=True)
    got = w.float().cpu().numpy()
    assert np.abs(got[:, :cols] - ref).max() <= 2 ** -7 * np.abs(ref).max() + 1e-30
    assert np.all(got[:, cols:] == 0)


def test_mix_one_hot_is_rounded_decode(cuda):
    """With p = e_k the mixture is exactly bf16(decode(W_k))."""
    from voodoo_quant import _C

    types = ["Q2_K", "Q6_K", "IQ4_XS"]
    _, cb = _cands(types, 40, 1024, seed=3)
    for k in range(3):
        p = torch.zeros(3)
        p[k] = 1.0
        w = _C.mix(types, [cb[q].to(cuda) for q in types], p.to(cuda), 40, 1024, 1024)
        ref = _C.dequant(cb[types[k]].to(cuda), types[k], 40, 1024).to(torch.bfloat16)
        assert torch.equal(w, ref)


def test_mix_full_size_and_unaligned_streams(cuda):
    """A config-2-sized mixture (14336 x 4096, six candidates: each persistent
    CTA walks many blocks, refilling its bulk-copy stages) against a float32
    torch mixture of the exact decodes (2^-7 of the largest weight); one-hot
    gates give bf16(decode) bit for bit; and candidate streams that start 2,
    6 or 10 bytes past a 16-byte boundary give the same bits as aligned ones."""
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn

    types = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]
    rows, cols = 14336, 4096
    g = torch.Generator(device=cuda).manual_seed(17)
    w = torch.randn(rows, cols, generator=g, device=cuda) * 0.02
    blocks = [rtn.quantize(w, q) for q in types]
    del w
    probs = torch.softmax(torch.randn(len(types), generator=g, device=cuda), 0)
    got = _C.mix(types, blocks, probs, rows, cols, cols)
    ref = torch.zeros(rows, cols, device=cuda)
    for k, (q, b) in enumerate(zip(types, blocks)):
        ref += probs[k] * _C.dequant(b, q, rows, cols)
    assert float((got.float() - ref).abs().max()) <= 2 ** -7 * float(ref.abs().max())
    for k in (1, 4):  # Q3_K and Q6_K: units that start inside a word
        one = torch.zeros(len(types), device=cuda)
        one[k] = 1.0
        w1 = _C.mix(types, blocks, one, rows, cols, cols)
        assert torch.equal(w1, _C.dequant(blocks[k], types[k], rows, cols).to(torch.bfloat16)), types[k]
    shifted = []
    for k, b in enumerate(blocks):
        off = (2, 6, 10)[k % 3]
        buf = torch.zeros(b.numel() + 32, dtype=torch.uint8, device=cuda)
        buf[off:off + b.numel()] = b.reshape(-1)
        shifted.append(buf[off:off + b.numel()])
    assert torch.equal(_C.mix(types, shifted, probs, rows, cols, cols), got)
    torch.cuda.synchronize()
    assert _C.device_error() == 0


def _bf16(t):
    return t.to(torch.bfloat16)


@pytest.mark.parametrize("T,N,K", [(128, 256, 64), (256, 512, 1024), (200, 384, 320), (1, 256, 256),
                                   (333, 1000, 776), (1024, 2048, 4096)])
def test_linear_fwd_dx_vs_torch(cuda, T, N, K):
    from voodoo_quant import _C

    torch.manual_seed(T + N + K)
    x = _bf16(torch.randn(T, K, device=cuda))
    w = _bf16(torch.randn(N, K, device=cuda) * 0.05)
    y = _C.linear_fwd(x, w)
    ref = x.float() @ w.float().T
    assert rel_err(y.float().cpu().numpy(), ref.cpu().numpy()) < TOL_GEMM
    dy = _bf16(torch.randn(T, N, device=cuda))
    dx = _C.linear_dx(dy, w, K)
    ref_dx = dy.float() @ w.float()
    assert rel_err(dx.float().cpu().numpy(), ref_dx.cpu().numpy()) < TOL_GEMM
    assert _C.device_error() == 0


def test_linear_fwd_exact_small_integers(cuda):
    """Integer-valued bf16 inputs make the fp32-accumulated product exact: any
    descriptor/swizzle/tile mistake shows up as a hard mismatch."""
    from voodoo_quant import _C

    g = torch.Generator(device="cpu").manual_seed(5)
    T, N, K = 384, 512, 512
    x = torch.randint(-3, 4, (T, K), generator=g).to(cuda, torch.bfloat16)
    w = torch.randint(-3, 4, (N, K), generator=g).to(cuda, torch.bfloat16)
    # the fp32 accumulation is exact, so the bf16 output is the single rounding of the exact product
    assert torch.equal(_C.linear_fwd(x, w), (x.double() @ w.double().T).to(torch.bfloat16))
    dy = torch.randint(-3, 4, (T, N), generator=g).to(cuda, torch.bfloat16)
    assert torch.equal(_C.linear_dx(dy, w, K), (dy.double() @ w.double()).to(torch.bfloat16))


@pytest.mark.parametrize("T,N,K,ld_pad,col_off", [(333, 1000, 512, 24, 0), (4100, 4096, 512, 64, 0),
                                                   (129, 256, 64, 8, 0), (257, 520, 128, 3, 0),
                                                   (300, 768, 192, 0, 1)])
def test_linear_store_edges_exact(cuda, T, N, K, ld_pad, col_off):
    """The paired store epilogue writes bulk tensor stores of 32 x 32 boxes
    where the output allows it (16-byte aligned base and row pitch) and row
    by row elsewhere (odd pitch, unaligned base): both against the exact
    product, with ragged last rows and columns, and every element outside
    the output (padding between rows, rows past its end) left untouched."""
    from voodoo_quant import _C

    g = torch.Generator(device="cpu").manual_seed(T + N + K + ld_pad)
    x = torch.randint(-3, 4, (T, K), generator=g).to(cuda, torch.bfloat16)
    w = torch.randint(-3, 4, (N, K), generator=g).to(cuda, torch.bfloat16)
    dy = torch.randint(-3, 4, (T, N), generator=g).to(cuda, torch.bfloat16)
    for width, fn, ref in ((N, lambda o: _C.linear_fwd(x, w, out=o), x.double() @ w.double().T),
                           (K, lambda o: _C.linear_dx(dy, w, K, out=o), dy.double() @ w.double())):
        big = torch.full((T + 40, width + ld_pad + col_off), float("inf"), dtype=torch.bfloat16, device=cuda)
        out = big[:T, col_off:col_off + width]
        fn(out)
        assert torch.equal(out, ref.to(torch.bfloat16))
        assert torch.isinf(big[:T, :col_off]).all() and torch.isinf(big[:T, col_off + width:]).all()
        assert torch.isinf(big[T:]).all()
    assert _C.device_error() == 0


@pytest.mark.parametrize("types,T,N,IN", [
    (["Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 1000, 1000, 1000),
    (["Q8_0"], 4096, 4096, 4096),
    (["IQ4_XS", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "Q2_K"], 300, 768, 512),
    (["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 2048, 1792, 4096),
])
def test_mixgemm_fwd_fused_equals_mix_then_gemm(cuda, types, T, N, IN):
    """The forward with the mixture decoded by producer warps into the GEMM's
    shared-memory operand tiles against the mix kernel followed by the plain
    GEMM: bit for bit (the same decode arithmetic, the same bf16 operand,
    the same tcgen05 accumulation), with ragged rows, columns and K and
    every candidate format."""
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn

    padded = (IN + 255) // 256 * 256
    g = torch.Generator(device="cpu").manual_seed(T + N + IN + len(types))
    w = torch.randn(N, padded, generator=g) * 0.02
    blocks = [rtn.quantize(w, q).to(cuda) for q in types]
    probs = torch.softmax(torch.randn(len(types), generator=g), 0).to(cuda)
    x = _bf16(torch.randn(T, IN, generator=g)).to(cuda)
    wm = _C.mix(types, blocks, probs, N, padded, IN)
    ref = _C.linear_fwd(x, wm, N, IN)
    got = _C.mixgemm_fwd_fused(x, types, blocks, probs, N, padded, IN)
    assert torch.equal(got, ref)
    assert _C.device_error() == 0


@pytest.mark.parametrize("T,F,K,ld_pad,col_off", [(300, 256, 512, 0, 0), (4096, 1792, 4096, 0, 0),
                                                   (1000, 1024, 1000, 16, 0), (257, 384, 256, 3, 1)])
def test_linear_fwd_swiglu_equals_gemm_then_swiglu(cuda, T, F, K, ld_pad, col_off):
    """The gate|up GEMM with the SwiGLU in its epilogue against the same GEMM
    into a bf16 [T, 2F] output followed by the SwiGLU kernel: bit for bit
    (ragged row and K tails, bulk stores and, for an unaligned output, row
    stores), with nothing written outside the output."""
    from voodoo_quant import _C

    g = torch.Generator(device="cpu").manual_seed(T + F + K)
    x = _bf16(torch.randn(T, K, generator=g)).to(cuda)
    w = _bf16(torch.randn(2 * F, K, generator=g) * 0.05).to(cuda)
    gu = _C.linear_fwd(x, w, 2 * F, K)
    ref = _C.swiglu_fwd(gu[:, :F], gu[:, F:])
    big = torch.full((T + 8, F + ld_pad + col_off), float("inf"), dtype=torch.bfloat16, device=cuda)
    out = big[:T, col_off:col_off + F]
    _C.linear_fwd_swiglu(x, w, F, K, out=out)
    assert torch.equal(out, ref)
    assert torch.isinf(big[T:]).all() and torch.isinf(big[:T, :col_off]).all()
    assert torch.isinf(big[:T, col_off + F:]).all()
    with pytest.raises(ValueError):
        _C.linear_fwd_swiglu(x[:, :K], w[: 2 * (F - 64)], F - 64, K)  # not a multiple of 128 features
    with pytest.raises(ValueError):
        _C.linear_fwd_swiglu(x[:128], w, F, K)  # 128 rows: no CTA-pair tile
    assert _C.device_error() == 0


@pytest.mark.parametrize("types,T,N,IN", [
    (["Q4_K", "Q5_K", "Q6_K", "Q8_0"], 256, 256, 512),
    (["Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 300, 200, 768),
    (["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 64, 130, 1000),
    (["IQ4_XS", "Q8_0"], 1, 128, 256),
])
def test_gategrad_matches_oracle(cuda, types, T, N, IN):
    from voodoo_quant import _C

    padded = (IN + 255) // 256 * 256
    _, cb = _cands(types, N, padded, seed=T)
    torch.manual_seed(N)
    x = _bf16(torch.randn(T, IN))
    dy = _bf16(torch.randn(T, N))
    g = _C.gategrad(dy.to(cuda), x.to(cuda), types, [cb[q].to(cuda) for q in types], N, IN, padded)
    cands = mixgemm.decode_candidates([cb[q].numpy() for q in types], types, N, padded, IN)
    ref = mixgemm.prob_grad(dy.float().numpy(), x.float().numpy(), cands, fp64=True)
    assert rel_err(g.cpu().numpy(), ref) < 1e-3
    assert _C.device_error() == 0


def test_gategrad_is_deterministic(cuda):
    from voodoo_quant import _C

    types = ["Q4_K", "Q6_K", "Q8_0"]
    _, cb = _cands(types, 512, 1024, seed=9)
    x = _bf16(torch.randn(700, 1024, device=cuda))
    dy = _bf16(torch.randn(700, 512, device=cuda))
    blocks = [cb[q].to(cuda) for q in types]
    a = _C.gategrad(dy, x, types, blocks, 512, 1024, 1024)
    b = _C.gategrad(dy, x, types, blocks, 512, 1024, 1024)
    assert torch.equal(a, b)


@pytest.mark.parametrize("case", ["k4", "k5", "k6"])
def test_module_matches_reference_golden(cuda, golden_dir, case):
    """MixedQuantLinear forward/backward vs the reference's own autograd outputs."""
    from voodoo_quant.layers import MixedQuantLinear

    z = np.load(golden_dir / "mixlinear_golden.npz")
    fmts = list(z[f"{case}/formats"])
    x = torch.from_numpy(z[f"{case}/x"])
    dy = torch.from_numpy(z[f"{case}/dy"])
    out_f, in_f = dy.shape[1], x.shape[1]
    cb = {q: torch.from_numpy(z[f"{case}/cand{k}/bytes"]).reshape(-1) for k, q in enumerate(fmts)}
    m = MixedQuantLinear(in_f, out_f, fmts, torch.zeros(out_f, in_f, device=cuda), candidate_bytes=cb,
                         tensor_name=f"golden.{case}")
    with torch.no_grad():
        m.gates.copy_(torch.from_numpy(z[f"{case}/gates"]))
    m.set_temperature(float(z[f"{case}/tau"]))
    xg = x.to(cuda).requires_grad_(True)
    y = m(xg)
    assert y.dtype == torch.float32
    y.backward(dy.to(cuda))
    assert rel_err(y.detach().cpu().numpy(), z[f"{case}/y"]) < TOL_GEMM
    assert rel_err(xg.grad.cpu().numpy(), z[f"{case}/dx"]) < TOL_GEMM
    assert cosine(m.gates.grad.cpu().numpy(), z[f"{case}/dgates"]) >= TOL_COS
    assert rel_err(m.gates.grad.cpu().numpy(), z[f"{case}/dgates"]) < 2e-2


def test_module_3d_input_and_empty_batch(cuda):
    from voodoo_quant.layers import MixedQuantLinear

    types = ["Q4_K", "Q8_0"]
    w, cb = _cands(types, 96, 256, seed=11)
    m = MixedQuantLinear(256, 96, types, w.to(cuda), candidate_bytes=cb, tensor_name="t.3d")
    x = _bf16(torch.randn(2, 5, 256, device=cuda)).requires_grad_(True)
    y = m(x)
    assert y.shape == (2, 5, 96)
    y.float().sum().backward()
    assert x.grad.shape == x.shape and m.gates.grad.shape == (2,)
    x0 = _bf16(torch.randn(0, 256, device=cuda)).requires_grad_(True)
    y0 = m(x0)
    assert y0.shape == (0, 96)
    y0.float().sum().backward()


def test_embedding_rows_match_oracle(cuda):
    from voodoo_quant.layers import MixedQuantEmbedding

    types = ["Q4_K", "Q6_K", "Q8_0"]
    V, D = 300, 512
    w, cb = _cands(types, V, D, seed=13)
    e = MixedQuantEmbedding(V, D, types, w.to(cuda), candidate_bytes=cb, tensor_name="emb")
    with torch.no_grad():
        e.gates.copy_(torch.tensor([0.3, -0.2, 0.5]))
    ids = torch.tensor([[5, 7, 5, 299], [0, 7, 123, 5]], device=cuda)
    out = e(ids)
    g = torch.randn(out.shape, device=cuda)
    (out.float() * g).sum().backward()
    p = torch.softmax(e.gates.detach().cpu(), 0).numpy()
    cands = mixgemm.decode_candidates([cb[q].numpy() for q in types], types, V, D, D)
    wm = mixgemm.mixed_weight(cands, p, fp64=True)
    ref = wm[ids.cpu().numpy()]
    assert rel_err(out.detach().float().cpu().numpy(), ref) < 1e-2
    gn = g.cpu().numpy()
    idn = ids.cpu().numpy()
    gp = np.array([np.sum(gn * c[idn]) for c in cands])
    ref_dg = mixgemm.gate_grad(p, gp, 1.0)
    assert cosine(e.gates.grad.cpu().numpy(), ref_dg) >= TOL_COS


@pytest.mark.parametrize("case", ["t1", "t2"])
def test_fused_loss_vs_reference_golden(cuda, golden_dir, case):
    from voodoo_quant.training.loss import distillation_loss

    z = np.load(golden_dir / "loss_golden.npz")
    s = torch.from_numpy(z[f"{case}/student"])
    V = s.shape[-1]
    sb = s.to(cuda, torch.bfloat16).requires_grad_(True)
    tb = torch.from_numpy(z[f"{case}/teacher"]).to(cuda, torch.bfloat16)
    y = torch.from_numpy(z[f"{case}/targets"]).to(cuda)
    loss, ce, kl = distillation_loss(sb, tb, y, float(z[f"{case}/temperature"]), 1.0, ce_reduction="tokens")
    loss.backward()
    # reference values come from fp32 logits; ours read the bf16-rounded logits
    ce_ref, kl_ref, g_ref = oloss.loss_and_grad(sb.detach().float().cpu().numpy().reshape(-1, V),
                                                tb.float().cpu().numpy().reshape(-1, V),
                                                y.cpu().numpy().reshape(-1), float(z[f"{case}/temperature"]))
    assert abs(ce.item() - ce_ref) < 1e-3 * abs(ce_ref)
    assert abs(kl.item() - kl_ref) < 1e-2 * abs(kl_ref) + 1e-4
    assert abs(ce.item() - float(z[f"{case}/ce"])) < 1e-2 * abs(float(z[f"{case}/ce"]))
    assert rel_err(sb.grad.float().cpu().numpy().reshape(-1, V), g_ref) < 1e-2


@pytest.mark.parametrize("V,temp", [(4096, 1.0), (50000, 2.0), (1001, 0.7), (152064, 1.0)])
def test_fused_loss_rows_vs_oracle(cuda, V, temp):
    from voodoo_quant import _C

    torch.manual_seed(V)
    rows = 24
    s = (torch.randn(rows, V, device=cuda) * 4).to(torch.bfloat16)
    t = (torch.randn(rows, V, device=cuda) * 4).to(torch.bfloat16)
    y = torch.randint(0, V, (rows,), device=cuda)
    y[3] = -100  # ignored target
    ce, kl, g = _C.loss_fused(s, t, y, temp, 1.0 / rows, 0.5 / rows)
    ce_r, kl_r = oloss.row_terms(s.float().cpu().numpy(), t.float().cpu().numpy(), y.cpu().numpy(), temp)
    assert ce[3].item() == 0.0
    assert rel_err(ce.cpu().numpy(), ce_r) < 1e-4
    assert rel_err(kl.cpu().numpy(), kl_r) < 1e-2
    _, _, g_r = oloss.loss_and_grad(s.float().cpu().numpy(), t.float().cpu().numpy(), y.cpu().numpy(), temp, 0.5)
    assert rel_err(g.float().cpu().numpy(), g_r) < 1e-2


def test_loss_vocab_parallel_combine_equals_fused(cuda):
    """Two vocabulary shards through stats -> combine -> grad equal the fused kernel."""
    from voodoo_quant import _C

    torch.manual_seed(2)
    rows, V, temp = 40, 6000, 1.5
    s = (torch.randn(rows, V, device=cuda) * 3).to(torch.bfloat16)
    t = (torch.randn(rows, V, device=cuda) * 3).to(torch.bfloat16)
    y = torch.randint(0, V, (rows,), device=cuda)
    ce, kl, g = _C.loss_fused(s, t, y, temp, 1.0 / rows, 1.0 / rows)
    cut = 2048  # uneven shards, multiple of 8
    st0 = _C.loss_stats(s[:, :cut].contiguous(), t[:, :cut].contiguous(), y, 0, temp)
    st1 = _C.loss_stats(s[:, cut:].contiguous(), t[:, cut:].contiguous(), y, cut, temp)
    lse, ce2, kl2 = _C.loss_combine(torch.stack([st0, st1]), temp)
    assert rel_err(ce2.cpu().numpy(), ce.cpu().numpy()) < 1e-5
    assert rel_err(kl2.cpu().numpy(), kl.cpu().numpy()) < 1e-4
    g0 = _C.loss_grad(s[:, :cut].contiguous(), t[:, :cut].contiguous(), y, 0, temp, lse, 1.0 / rows, 1.0 / rows)
    g1 = _C.loss_grad(s[:, cut:].contiguous(), t[:, cut:].contiguous(), y, cut, temp, lse, 1.0 / rows, 1.0 / rows)
    gg = torch.cat([g0, g1], 1).float()
    assert rel_err(gg.cpu().numpy(), g.float().cpu().numpy()) < 1e-2


# ----------------------------------------------------------------- full-size properties
def test_config2_shapes_properties(cuda):
    """BASELINE config-2 shapes (T=8192, N=14336, Kin=4096, K=5): forward against
    torch's fp32 product of the same bf16 operands (sampled rows), gate-gradient
    linearity in dY, and one-hot-gate equivalence of mix and decode."""
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn

    types = ["Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]
    T, N, IN = 8192, 14336, 4096
    g = torch.Generator(device=cuda).manual_seed(0)
    w = torch.randn(N, IN, device=cuda, generator=g) * 0.02
    blocks = [rtn.quantize(w, q).contiguous() for q in types]
    del w
    probs = torch.softmax(torch.randn(len(types), device=cuda, generator=g) / 0.5, 0)
    wm = _C.mix(types, blocks, probs, N, IN, IN)
    x = torch.randn(T, IN, device=cuda, generator=g).to(torch.bfloat16)
    y = _C.linear_fwd(x, wm)
    rows = torch.randint(0, T, (64,), device=cuda, generator=g)
    ref = x[rows].float() @ wm.float().T
    assert rel_err(y[rows].float().cpu().numpy(), ref.cpu().numpy()) < 5e-3
    dy1 = torch.randn(T, N, device=cuda, generator=g).to(torch.bfloat16)
    dy2 = torch.randn(T, N, device=cuda, generator=g).to(torch.bfloat16)
    cols = torch.randint(0, IN, (64,), device=cuda, generator=g)
    dx = _C.linear_dx(dy1, wm, IN)
    ref_dx = dy1[:256].float() @ wm.float()
    assert rel_err(dx[:256].float().cpu().numpy(), ref_dx.cpu().numpy()) < 5e-3
    del cols
    ga = _C.gategrad(dy1, x, types, blocks, N, IN, IN)
    gb = _C.gategrad(dy2, x, types, blocks, N, IN, IN)
    gs = _C.gategrad((dy1.float() + dy2.float()).to(torch.bfloat16), x, types, blocks, N, IN, IN)
    assert rel_err(gs.cpu().numpy(), (ga + gb).cpu().numpy()) < 2e-2
    # reference gate gradient for one candidate through torch's fp32 dW of a row band
    band = slice(0, 512)
    w0 = _C.dequant(blocks[0].view(N, -1)[band].reshape(-1, 110), "Q3_K", 512, IN)
    xs, ds = x[:2048].float(), dy1[:2048, band].float()
    gpart = _C.gategrad(dy1[:2048, band].contiguous(), x[:2048].contiguous(), ["Q3_K"],
                        [blocks[0].view(N, -1)[band].reshape(-1, 110).contiguous()], 512, IN, IN)
    ref_part = ((ds.T @ xs) * w0).sum()
    assert abs(gpart.item() - ref_part.item()) <= 1e-3 * abs(ref_part.item()) + 1e-3
    assert _C.device_error() == 0


@pytest.mark.parametrize("T,N,IN", [(1024, 2560, 2048), (640, 14336, 512), (2048, 512, 4096), (1000, 768, 2048),
                                    (4096, 128, 4096)])
def test_gategrad_stream_k_tail_matches_fp64(cuda, T, N, IN):
    """Shapes whose tile count is not a multiple of the CTA-pair count, so the
    last wave is split along K (stream-K pieces writing their own partial
    slots), and shapes with at most half as many tiles as pairs, where every
    tile is split (two or three row blocks walking the same column ranges
    together, or one): against fp64 <dy^T x, W_k> with W_k decoded
    bit-exactly."""
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn

    types = ["Q3_K", "Q4_K", "Q6_K", "Q8_0"]
    g = torch.Generator(device="cpu").manual_seed(N + IN)
    w = torch.randn(N, IN, generator=g) * 0.02
    blocks = [rtn.quantize(w, q).to(cuda) for q in types]
    x = _bf16(torch.randn(T, IN, generator=g)).to(cuda)
    dy = _bf16(torch.randn(T, N, generator=g)).to(cuda)
    dw = dy.double().T @ x.double()
    ref = torch.stack([(dw * _C.dequant(b, q, N, IN).double()).sum() for q, b in zip(types, blocks)])
    got = _C.gategrad(dy, x, types, blocks, N, IN, IN)
    assert rel_err(got.double().cpu().numpy(), ref.cpu().numpy()) < 1e-3
    assert torch.equal(got, _C.gategrad(dy, x, types, blocks, N, IN, IN))
    assert _C.device_error() == 0


@pytest.mark.parametrize("T,rows,IN", [(2048, (512, 128, 128), 4096), (1000, (1792, 1792), 2048),
                                       (300, (256, 32), 512)])
def test_gategrad_grouped_matches_fp64(cuda, T, rows, IN):
    """Layers side by side in dY's columns (q/k/v, gate/up) through one
    grouped gate-gradient GEMM: each layer's gradients against fp64
    <dy_g^T x, W_{g,k}> (1e-3 relative), written `ld` floats apart into a
    wider buffer whose other entries stay untouched, and within 1e-4 of
    the per-layer launches (fp32 partial sums split differently along K)."""
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn

    types = ["Q3_K", "Q4_K", "Q6_K", "Q8_0"]
    g = torch.Generator(device="cpu").manual_seed(T + IN)
    blocks = []
    for n in rows:
        w = torch.randn(n, IN, generator=g) * 0.02
        blocks.append([rtn.quantize(w, q).to(cuda) for q in types])
    x = _bf16(torch.randn(T, IN, generator=g)).to(cuda)
    dy = _bf16(torch.randn(T, sum(rows), generator=g)).to(cuda)
    buf = torch.full((len(rows), 8), 7.0, device=cuda)
    got = _C.gategrad_grouped(dy, x, types, blocks, list(rows), IN, IN, out=buf[:, :len(types)])
    assert torch.all(buf[:, len(types):] == 7.0)
    a = 0
    for i, n in enumerate(rows):
        dw = dy[:, a:a + n].double().T @ x.double()
        ref = torch.stack([(dw * _C.dequant(b, q, n, IN).double()).sum() for q, b in zip(types, blocks[i])])
        assert rel_err(got[i].double().cpu().numpy(), ref.cpu().numpy()) < 1e-3, i
        one = _C.gategrad(dy[:, a:a + n], x, types, blocks[i], n, IN, IN)
        assert rel_err(got[i].cpu().numpy(), one.cpu().numpy()) < 1e-4, i
        a += n
    assert torch.equal(got, _C.gategrad_grouped(dy, x, types, blocks, list(rows), IN, IN))
    with pytest.raises(ValueError):
        _C.gategrad_grouped(dy[:, :sum(rows) - 16], x, types, blocks, [rows[0], rows[1] - 16] + list(rows[2:]), IN, IN)
    assert _C.device_error() == 0


def test_sm_reserve_keeps_results(cuda):
    """GEMMs that leave SMs free for a concurrent collective
    (vq_set_gemm_sm_reserve, vq_set_gategrad_sm_reserve) compute the same
    tiles with fewer CTAs: forward and dX bit-identical, gate gradients within
    1e-3 relative (the stream-K split of the last wave changes with the CTA
    count, so fp32 partial sums are added in another order)."""
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn

    types = ["Q4_K", "Q6_K", "Q8_0"]
    T, N, IN = 2048, 3584, 4096
    g = torch.Generator(device="cpu").manual_seed(17)
    w = torch.randn(N, IN, generator=g) * 0.02
    blocks = [rtn.quantize(w, q).to(cuda) for q in types]
    x = _bf16(torch.randn(T, IN, generator=g)).to(cuda)
    dy = _bf16(torch.randn(T, N, generator=g)).to(cuda)
    wm = _bf16(w).to(cuda)
    base = (_C.linear_fwd(x, wm, N, IN), _C.linear_dx(dy, wm, IN), _C.gategrad(dy, x, types, blocks, N, IN, IN))
    try:
        _C.set_gemm_sm_reserve(24)
        _C.set_gategrad_sm_reserve(24)
        res = (_C.linear_fwd(x, wm, N, IN), _C.linear_dx(dy, wm, IN), _C.gategrad(dy, x, types, blocks, N, IN, IN))
    finally:
        _C.set_gemm_sm_reserve(0)
        _C.set_gategrad_sm_reserve(0)
    assert torch.equal(base[0], res[0]) and torch.equal(base[1], res[1])
    # fewer clusters split the last wave's k-blocks differently: fp32 sums in another order
    assert rel_err(res[2].double().cpu().numpy(), base[2].double().cpu().numpy()) < 1e-3
    with pytest.raises(ValueError):
        _C.set_gemm_sm_reserve(-1)
    assert _C.device_error() == 0
