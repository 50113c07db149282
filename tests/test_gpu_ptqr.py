"""PTQR (per-token quant routing) on the B200 kernels against the reference's
own routed functions (tests/golden/ptqr_golden.npz, a fixed routing):

* linear: y, dX within 1e-2 relative of the reference's float32 (bf16 GEMM);
  gate gradients cosine >= 0.999 and within 2e-2 relative;
* embedding rows: equal values, bit-identical except the sign of zero (exact
  decode of the routed candidate, rounded once to bf16); d probs within 1e-2
  relative (the reference forms the products in bf16).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cosine, rel_err

pytestmark = pytest.mark.gpu


def _linear(z, cuda):
    from voodoo_quant.layers import MixedQuantLinear

    fmts = [str(f) for f in z["lin/formats"]]
    out_f, in_f = z["lin/dy"].shape[1], z["lin/x"].shape[1]
    cb = {q: torch.from_numpy(z[f"lin/cand{k}/bytes"]).reshape(-1) for k, q in enumerate(fmts)}
    m = MixedQuantLinear(in_f, out_f, fmts, torch.zeros(out_f, in_f, device=cuda), candidate_bytes=cb,
                         tensor_name="golden.ptqr.lin")
    with torch.no_grad():
        m.gates.copy_(torch.from_numpy(z["lin/gates"]))
    m.set_temperature(float(z["lin/tau"]))
    return m


def test_routed_linear_matches_reference(cuda, golden_dir):
    from voodoo_quant.layers import _RoutedGatedLinearFunction

    z = np.load(golden_dir / "ptqr_golden.npz")
    m = _linear(z, cuda)
    x = torch.from_numpy(z["lin/x"]).to(cuda).requires_grad_(True)
    routing = torch.from_numpy(z["lin/routing"]).to(cuda)
    y = _RoutedGatedLinearFunction.apply(x, m.get_probs(), m, routing)
    y.backward(torch.from_numpy(z["lin/dy"]).to(cuda))
    assert rel_err(y.detach().cpu().numpy(), z["lin/y"]) < 1e-2
    assert rel_err(x.grad.cpu().numpy(), z["lin/dx"]) < 1e-2
    g = m.gates.grad.cpu().numpy()
    assert cosine(g, z["lin/dgates"]) >= 0.999 and rel_err(g, z["lin/dgates"]) < 2e-2


def test_ptqr_switch_routes_every_token_to_one_candidate(cuda, golden_dir):
    """With set_ptqr(True) the module samples a routing; each output row is
    exactly that row's GEMM against one candidate (checked against the fixed-
    routing function on the sampled routing), and the backward is the
    mixture's."""
    from voodoo_quant.layers import _RoutedGatedLinearFunction, _sample_token_routing, set_ptqr

    z = np.load(golden_dir / "ptqr_golden.npz")
    m = _linear(z, cuda)
    x = torch.from_numpy(z["lin/x"]).to(cuda, torch.bfloat16)
    try:
        set_ptqr(True)
        torch.manual_seed(7)
        y = m(x)
    finally:
        set_ptqr(False)
    torch.manual_seed(7)
    routing = _sample_token_routing(m.get_probs().to(cuda), x.shape[0])
    assert routing.unique().numel() > 1
    ref = _RoutedGatedLinearFunction.apply(x, m.get_probs(), m, routing)
    assert torch.equal(y, ref)
    y_mix = m(x)  # PTQR off again: the mixture forward
    assert not torch.equal(y_mix, y)


def test_routed_embedding_rows_match_reference(cuda, golden_dir):
    from voodoo_quant.layers import MixedQuantEmbedding, _GatedEmbeddingRowsFunction

    z = np.load(golden_dir / "ptqr_golden.npz")
    fmts = [str(f) for f in z["lin/formats"]]
    V, D = 64, 512
    cb = {q: torch.from_numpy(z[f"emb/cand{k}/bytes"]).reshape(-1) for k, q in enumerate(fmts)}
    e = MixedQuantEmbedding(V, D, fmts, torch.zeros(V, D, dtype=torch.bfloat16, device=cuda), candidate_bytes=cb,
                            tensor_name="golden.ptqr.emb")
    probs = torch.softmax(torch.from_numpy(z["emb/gates"]).to(cuda), 0).detach().requires_grad_(True)
    rows = torch.from_numpy(z["emb/row_ids"]).to(cuda)
    out = _GatedEmbeddingRowsFunction.apply(probs, rows, e, torch.from_numpy(z["emb/routing"]).to(cuda))
    assert out.dtype == torch.bfloat16
    # equal values (the mixture kernel's fp32 accumulation starts from +0, so an
    # exact -0 decode comes out as +0; every other value is bit-identical)
    got = out.detach().float().cpu().numpy()
    assert np.array_equal(got, z["emb/rows"])
    nz = got != 0
    assert np.array_equal(got[nz].view(np.uint32), z["emb/rows"][nz].view(np.uint32))
    out.float().backward(torch.from_numpy(z["emb/grad_out"]).to(cuda))
    assert rel_err(probs.grad.cpu().numpy(), z["emb/dprobs"]) < 1e-2


@pytest.mark.parametrize("sizes", [[300, 0, 129, 1], [0, 0, 700, 0], [256, 256, 257, 255], [5, 1000, 3, 2, 40, 0, 7, 500]])
def test_grouped_gemm_matches_per_group_gemms(cuda, sizes):
    """vq_linear_fwd_grouped against one plain GEMM per group, bit for bit
    (same tcgen05 tiles and accumulation order), with empty groups."""
    from voodoo_quant import _C

    g = torch.Generator(device="cpu").manual_seed(sum(sizes))
    T, K, N = sum(sizes), 512, 768
    x = torch.randn(T, K, generator=g).to(cuda, torch.bfloat16)
    ws = [(torch.randn(N, K, generator=g) * 0.05).to(cuda, torch.bfloat16) for _ in sizes]
    off = torch.tensor([0] + list(np.cumsum(sizes)), dtype=torch.int32, device=cuda)
    y = _C.linear_fwd_grouped(x, ws, N, K, off)
    for i, n in enumerate(sizes):
        if n:
            a, b = int(off[i]), int(off[i + 1])
            ref = _C.linear_fwd(x[a:b].contiguous(), ws[i], N, K) if n > 128 else \
                (x[a:b].float() @ ws[i].float().T).to(torch.bfloat16)
            if n > 128:
                assert torch.equal(y[a:b], ref)
            else:
                assert rel_err(y[a:b].float().cpu().numpy(), ref.float().cpu().numpy()) < 1e-2
    assert _C.device_error() == 0


@pytest.mark.parametrize("T,K", [(1, 4), (1000, 3), (16384, 6), (70001, 8)])
def test_route_prep_is_a_stable_grouping(cuda, T, K):
    from voodoo_quant import _C

    g = torch.Generator(device="cpu").manual_seed(T + K)
    keys = torch.randint(0, K, (T,), generator=g, dtype=torch.int64)
    keys[: T // 3] = K - 1  # a skewed group
    order, inv, off = _C.route_prep(keys.to(cuda), K)
    ref = torch.argsort(keys, stable=True)
    assert torch.equal(order.cpu(), ref)
    assert torch.equal(inv.cpu()[ref], torch.arange(T))
    counts = torch.bincount(keys, minlength=K)
    assert torch.equal(off.cpu().long(), torch.cat([torch.zeros(1, dtype=torch.long), counts.cumsum(0)]))


def test_bank_routing_never_picks_padding(cuda):
    """Batched per-step routing for layers with different candidate counts:
    only valid candidates, and shares that follow each layer's probabilities."""
    from voodoo_quant.layers import GateBank, MixedQuantLinear
    from voodoo_quant.quants import rtn

    mods = {}
    for i, types in enumerate([("Q4_K", "Q8_0"), ("Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0")]):
        w = torch.randn(16, 256) * 0.02
        m = MixedQuantLinear(256, 16, list(types), w.to(cuda), candidate_bytes={q: rtn.quantize(w, q) for q in types},
                             tensor_name=f"bank.route.{i}")
        with torch.no_grad():
            m.gates.copy_(torch.linspace(-1, 1, len(types)))
        mods[f"l{i}"] = m
    bank = GateBank(mods)
    bank.probs()
    torch.manual_seed(0)
    for m in mods.values():
        r = bank.routing(m, 200000).long()
        assert int(r.max()) < m.num_candidates
        shares = torch.bincount(r, minlength=m.num_candidates).double().cpu() / r.numel()
        assert torch.allclose(shares, m.get_probs().double().cpu(), atol=6e-3)
    bank.release()
