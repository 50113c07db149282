"""Fused Llama-block kernels (RMSNorm, rotary embedding, SwiGLU) through the
C ABI against plain PyTorch fp32 references of the same ops, forward and
backward, and a patched model against the unpatched Hugging Face model.

Tolerance: 1e-2 relative (L2) for every bf16 output against the fp32
reference; bf16 results of the same op differ by at most one or two roundings.
"""

from __future__ import annotations

import pytest
import torch

from conftest import cosine, rel_err

pytestmark = pytest.mark.gpu


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return rel_err(a.detach().float().cpu().numpy(), b.detach().float().cpu().numpy())


def _rms_ref(x, w, eps):
    return w.float() * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


@pytest.mark.parametrize("rows,D", [(1, 1024), (37, 1024), (300, 4096), (64, 5120), (5, 8192), (3, 8)])
def test_rmsnorm_forward_backward(cuda, rows, D):
    from voodoo_quant import _C

    g = torch.Generator(device="cpu").manual_seed(rows * 7 + D)
    x = (torch.randn(rows, D, generator=g) * 3).to(cuda, torch.bfloat16)
    w = (1 + 0.3 * torch.randn(D, generator=g)).to(cuda, torch.bfloat16)
    dy = torch.randn(rows, D, generator=g).to(cuda, torch.bfloat16)
    y, rstd = _C.rmsnorm_fwd(x, w, 1e-6)
    xf = x.float().requires_grad_(True)
    yr = _rms_ref(xf, w, 1e-6)
    assert _rel(y, yr.detach()) < 1e-2
    assert torch.allclose(rstd, torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6), rtol=1e-5)
    yr.backward(dy.float())
    dx = _C.rmsnorm_bwd(x, dy, w, rstd)
    assert _rel(dx, xf.grad) < 1e-2


@pytest.mark.parametrize("rows,D", [(1, 1024), (300, 4096), (64, 5120), (3, 8)])
def test_add_rmsnorm_forward_backward(cuda, rows, D):
    """Residual add fused into RMSNorm: h is the bf16 sum torch computes, y is
    RMSNorm(h) bit for bit, and the input gradient is RMSNorm'(dy) + dh
    (fp32 sum, one rounding) within 1e-2 of an fp32 reference."""
    from voodoo_quant import _C
    from voodoo_quant.fused_blocks import add_rms_norm

    g = torch.Generator(device="cpu").manual_seed(rows * 11 + D)
    a = (torch.randn(rows, D, generator=g) * 2).to(cuda, torch.bfloat16)
    res = (torch.randn(rows, D, generator=g) * 3).to(cuda, torch.bfloat16)
    w = (1 + 0.3 * torch.randn(D, generator=g)).to(cuda, torch.bfloat16)
    h, y, rstd = _C.add_rmsnorm_fwd(a, res, w, 1e-6)
    assert torch.equal(h, a + res)
    y1, rstd1 = _C.rmsnorm_fwd(h, w, 1e-6)
    assert torch.equal(y, y1) and torch.equal(rstd, rstd1)
    dy = torch.randn(rows, D, generator=g).to(cuda, torch.bfloat16)
    dh = torch.randn(rows, D, generator=g).to(cuda, torch.bfloat16)
    dx = _C.rmsnorm_bwd_add(h, dy, dh, w, rstd)
    hf = h.float().requires_grad_(True)
    _rms_ref(hf, w, 1e-6).backward(dy.float())
    assert _rel(dx, hf.grad + dh.float()) < 1e-2
    # through autograd: both inputs receive the same gradient
    af, rf = a.clone().requires_grad_(True), res.clone().requires_grad_(True)
    hh, yy = add_rms_norm(af, rf, w, 1e-6)
    torch.autograd.backward([hh, yy], [dh, dy])
    assert torch.equal(af.grad, dx) and torch.equal(rf.grad, dx)


@pytest.mark.parametrize("B,S,Hq,Hk,D", [(2, 33, 4, 2, 128), (1, 8, 3, 1, 64), (2, 16, 8, 8, 16)])
def test_rope_forward_backward(cuda, B, S, Hq, Hk, D):
    from voodoo_quant import _C

    g = torch.Generator(device="cpu").manual_seed(B * 100 + S + D)
    # q/k as the attention builds them: views of a projection output [B, S, H * D]
    q = torch.randn(B, S, Hq * D, generator=g).to(cuda, torch.bfloat16).view(B, S, Hq, D)
    k = torch.randn(B, S, Hk * D, generator=g).to(cuda, torch.bfloat16).view(B, S, Hk, D)
    ang = torch.randn(B, S, D // 2, generator=g) * 3
    cos = torch.cat([ang.cos(), ang.cos()], -1).to(cuda, torch.bfloat16)
    sin = torch.cat([ang.sin(), ang.sin()], -1).to(cuda, torch.bfloat16)

    def ref(t):
        h = t.shape[-1] // 2
        rot = torch.cat([-t[..., h:], t[..., :h]], -1)
        return t * cos.float()[:, :, None] + rot * sin.float()[:, :, None]

    qf, kf = q.float().requires_grad_(True), k.float().requires_grad_(True)
    qr, kr = ref(qf), ref(kf)
    qo, ko = _C.rope(q, k, cos, sin)
    assert qo.is_contiguous() and qo.shape == q.shape
    assert _rel(qo, qr.detach()) < 1e-2 and _rel(ko, kr.detach()) < 1e-2
    gq = torch.randn(B, Hq, S, D, generator=g).to(cuda, torch.bfloat16).transpose(1, 2)  # SDPA-like layout
    gk = torch.randn(B, Hk, S, D, generator=g).to(cuda, torch.bfloat16).transpose(1, 2)
    torch.autograd.backward([qr, kr], [gq.float(), gk.float()])
    dq, dk = _C.rope(gq, gk, cos, sin, backward=True)
    assert _rel(dq, qf.grad) < 1e-2 and _rel(dk, kf.grad) < 1e-2


@pytest.mark.parametrize("rows,F", [(1, 8), (129, 3072), (64, 14336)])
def test_swiglu_forward_backward(cuda, rows, F):
    from voodoo_quant import _C

    g = torch.Generator(device="cpu").manual_seed(rows + F)
    a = (torch.randn(rows, F, generator=g) * 2).to(cuda, torch.bfloat16)
    u = torch.randn(rows, F, generator=g).to(cuda, torch.bfloat16)
    dy = torch.randn(rows, F, generator=g).to(cuda, torch.bfloat16)
    af, uf = a.float().requires_grad_(True), u.float().requires_grad_(True)
    yr = torch.nn.functional.silu(af) * uf
    assert _rel(_C.swiglu_fwd(a, u), yr.detach()) < 1e-2
    yr.backward(dy.float())
    da, du = _C.swiglu_bwd(a, u, dy)
    assert _rel(da, af.grad) < 1e-2 and _rel(du, uf.grad) < 1e-2


def test_block_kernels_reject_bad_shapes(cuda):
    from voodoo_quant import _C

    lib = _C.load_library()
    x = torch.zeros(4, 12, dtype=torch.bfloat16, device=cuda)
    w = torch.ones(12, dtype=torch.bfloat16, device=cuda)
    rc = lib.vq_rmsnorm_fwd(x.data_ptr(), 12, 4, 12, w.data_ptr(), 1e-6, x.data_ptr(), 12, None, None)
    assert rc == _C.VQ_ERR_INVALID and b"multiple of 8" in lib.vq_last_error()
    with pytest.raises(ValueError, match="multiple of 16"):
        q = torch.zeros(1, 2, 1, 8, dtype=torch.bfloat16, device=cuda)
        _C.rope(q, q, q[0, :, 0], q[0, :, 0])


def test_fused_llama_blocks_match_unpatched_model(cuda):
    from voodoo_quant.fused_blocks import fuse_llama_blocks
    from voodoo_quant.training import synthetic as S

    shape = S.ModelShape(2, 512, 4, 2, 1536, 2048, False, head_dim=128, batch=2, seq=64)
    ref = S.build_llama(shape, cuda, seed=4)
    fused = S.build_llama(shape, cuda, seed=4)
    # per layer: two norms, attention, MLP and the decoder layer (add + norm); plus the final norm
    assert fuse_llama_blocks(fused) == 2 * 5 + 1 and fuse_llama_blocks(fused) == 0
    x, _ = S.random_tokens(shape, cuda, seed=5)
    e_ref = ref.model.embed_tokens(x).detach().requires_grad_(True)
    e_fus = e_ref.detach().clone().requires_grad_(True)
    l_ref = ref(inputs_embeds=e_ref, use_cache=False).logits
    l_fus = fused(inputs_embeds=e_fus, use_cache=False).logits
    assert _rel(l_fus, l_ref) < 1e-2
    gy = torch.randn_like(l_ref)
    l_ref.backward(gy)
    l_fus.backward(gy)
    assert _rel(e_fus.grad, e_ref.grad) < 2e-2
    assert cosine(e_fus.grad.double().flatten().cpu().numpy(), e_ref.grad.double().flatten().cpu().numpy()) > 0.999


def test_chained_residual_adds_match_layer_by_layer(cuda):
    """With causal_batches the LlamaModel forward hands each layer's MLP
    output to the next RMSNorm unsummed (one add + norm kernel): logits
    bit-identical to the layer-by-layer fused forward (the same bf16 sums and
    norms), the embedding's gradient within bf16 rounding of it (the two
    gradient branches of a residual sum added in fp32 before one rounding),
    and both close to the unpatched Hugging Face model."""
    from voodoo_quant.fused_blocks import fuse_llama_blocks
    from voodoo_quant.training import synthetic as S

    shape = S.ModelShape(3, 512, 4, 2, 1536, 2048, False, head_dim=128, batch=2, seq=64)
    ref = S.build_llama(shape, cuda, seed=4)
    m = S.build_llama(shape, cuda, seed=4)
    assert fuse_llama_blocks(m, causal_batches=True) == 3 * 5 + 1 + 1
    x, _ = S.random_tokens(shape, cuda, seed=5)
    gy = torch.randn(shape.batch, shape.seq, shape.vocab, generator=torch.Generator(device=cuda).manual_seed(6),
                     device=cuda)

    def run(model):
        model.zero_grad(set_to_none=True)
        logits = model(input_ids=x, use_cache=False).logits
        logits.backward(gy.to(logits.dtype))
        return logits.detach(), model.model.embed_tokens.weight.grad.detach().clone()

    l_chain, g_chain = run(m)
    chained = m.model.forward
    m.model.forward = m.model._vq_chain_orig_forward
    try:
        l_layer, g_layer = run(m)
    finally:
        m.model.forward = chained
    l_ref, g_ref = run(ref)
    assert torch.equal(l_chain, l_layer)
    assert _rel(g_chain, g_layer) < 1e-2
    assert _rel(l_chain, l_ref) < 1e-2 and _rel(g_chain, g_ref) < 2e-2
    assert cosine(g_chain.double().flatten().cpu().numpy(), g_ref.double().flatten().cpu().numpy()) > 0.999


def _gated(cuda, n_out, n_in, types, seed):
    from voodoo_quant.layers import MixedQuantLinear
    from voodoo_quant.quants import rtn

    g = torch.Generator(device="cpu").manual_seed(seed)
    w = torch.randn(n_out, n_in, generator=g) * 0.02
    layer = MixedQuantLinear(n_in, n_out, types, w.to(cuda), candidate_bytes={q: rtn.quantize(w, q) for q in types},
                             tensor_name=f"group.{seed}")
    with torch.no_grad():
        layer.gates.copy_(torch.randn(len(types), generator=g))
    layer.set_temperature(0.7)
    return layer


@pytest.mark.parametrize("outs", [(512, 128, 128), (1792, 1792)])
def test_grouped_gated_projection_matches_separate_layers(cuda, outs):
    """q/k/v (or gate/up) as one grouped GEMM: the output columns equal each
    layer's own forward (the same mixture and dot products per output
    element; 1e-3 relative), dX equals the sum of the layers' dX within bf16
    rounding of the partial sums (1e-2 relative), and the layers' gate
    gradients, from one grouped gate-gradient GEMM, equal each layer's own
    within the order of fp32 partial sums (1e-4 relative)."""
    from voodoo_quant.layers import gated_linear_group, groupable

    types = ["Q2_K", "Q4_K", "Q6_K", "Q8_0"]
    n_in, T = 1024, 300
    layers = [_gated(cuda, n, n_in, types, 40 + i) for i, n in enumerate(outs)]
    assert groupable(layers)
    g = torch.Generator(device="cpu").manual_seed(9)
    x = torch.randn(T, n_in, generator=g).to(cuda, torch.bfloat16)
    dy = torch.randn(T, sum(outs), generator=g).to(cuda, torch.bfloat16)

    xa = x.clone().requires_grad_(True)
    ya = gated_linear_group(layers, xa)
    ya.backward(dy)
    ga = [l.gates.grad.clone() for l in layers]
    for l in layers:
        l.gates.grad = None

    xb = x.clone().requires_grad_(True)
    yb = torch.cat([l(xb) for l in layers], dim=1)
    yb.backward(dy)
    gb = [l.gates.grad.clone() for l in layers]
    torch.cuda.synchronize()
    assert _rel(ya, yb) < 1e-3
    assert _rel(xa.grad, xb.grad) < 1e-2
    for a, b in zip(ga, gb):
        assert _rel(a, b) < 1e-4


def test_grouped_q8_teacher_projection_matches_separate_layers(cuda):
    from voodoo_quant.quants import rtn
    from voodoo_quant.training.q8_teacher import Q8Linear, q8_groupable, q8_linear_group

    g = torch.Generator(device="cpu").manual_seed(11)
    mods = []
    for n in (512, 128, 128):
        w = torch.randn(n, 768, generator=g) * 0.02
        mods.append(Q8Linear(rtn.quantize(w, "Q8_0").to(cuda), n, 768))
    assert q8_groupable(mods)
    x = torch.randn(2, 70, 768, generator=g).to(cuda, torch.bfloat16)
    y = q8_linear_group(mods, x)
    assert y.shape == (2, 70, 768)
    assert _rel(y, torch.cat([m(x) for m in mods], dim=-1)) < 1e-3


def test_teacher_mlp_swiglu_in_the_gemm_epilogue(cuda):
    """A forward-only (teacher) MLP runs gate|up and the SwiGLU as one GEMM:
    equal, bit for bit, to the grouped gate|up GEMM followed by the SwiGLU
    kernel, and the fused MLP module takes that path under no_grad."""
    from voodoo_quant.fused_blocks import _SwiGLUPairFn, _mlp_forward
    from voodoo_quant.quants import rtn
    from voodoo_quant.training.q8_teacher import Q8Linear, q8_linear_group, q8_swiglu_group, q8_swiglu_ok

    g = torch.Generator(device="cpu").manual_seed(13)
    mods = []
    for n, k in ((1024, 768), (1024, 768), (768, 1024)):
        w = torch.randn(n, k, generator=g) * 0.02
        mods.append(Q8Linear(rtn.quantize(w, "Q8_0").to(cuda), n, k))
    gate, up, down = mods
    x = torch.randn(2, 150, 768, generator=g).to(cuda, torch.bfloat16)
    assert q8_swiglu_ok(gate, up, x)
    h = q8_swiglu_group(gate, up, x)
    ref = _SwiGLUPairFn.apply(q8_linear_group((gate, up), x))
    assert h.shape == (2, 150, 1024) and torch.equal(h, ref)

    class _MLP(torch.nn.Module):
        pass

    mlp = _MLP()
    mlp.gate_proj, mlp.up_proj, mlp.down_proj = gate, up, down
    with torch.no_grad():
        y = _mlp_forward(mlp, x)
    assert torch.equal(y, down(ref))
    assert not q8_swiglu_ok(gate, up, x[:, :60])  # 120 tokens: below one CTA-pair tile


def test_swiglu_pair_backward_layout(cuda):
    """The grouped gate|up SwiGLU writes d gate | d up side by side."""
    from voodoo_quant import _C
    from voodoo_quant.fused_blocks import _SwiGLUPairFn

    g = torch.Generator(device="cpu").manual_seed(12)
    gu = torch.randn(3, 50, 2 * 1792, generator=g).to(cuda, torch.bfloat16).requires_grad_(True)
    dy = torch.randn(3, 50, 1792, generator=g).to(cuda, torch.bfloat16)
    y = _SwiGLUPairFn.apply(gu)
    y.backward(dy)
    a, u = gu.detach()[..., :1792].reshape(-1, 1792), gu.detach()[..., 1792:].reshape(-1, 1792)
    assert torch.equal(y.reshape(-1, 1792), _C.swiglu_fwd(a, u))
    da, du = _C.swiglu_bwd(a, u, dy.reshape(-1, 1792))
    assert torch.equal(gu.grad.reshape(-1, 2 * 1792), torch.cat([da, du], dim=1))
