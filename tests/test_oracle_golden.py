"""The CPU oracle against vectors produced by the reference itself (tests/golden).

Pins the oracle before it is used as the checker for the CUDA path:
bit-exact block decoding for all seven formats (including +-0, subnormal,
65504, +-inf and NaN fp16 scales), the mixture/GEMM/gate-gradient math of
``_MixedWeightFunction`` + ``F.linear`` and the chunked CE + KL loss.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_err, same_bits
from oracle import ggml_blocks, loss as oloss, mixgemm

FORMATS = list(ggml_blocks.FORMATS)


@pytest.fixture(scope="module")
def dq(golden_dir):
    return np.load(golden_dir / "dequant_golden.npz")


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("tag", ["regular", "edge"])
def test_dequant_bit_exact(dq, fmt, tag):
    raw = dq[f"{fmt}/{tag}/bytes"]
    exp = dq[f"{fmt}/{tag}/expected"]
    got = ggml_blocks.dequantize(raw, fmt, exp.shape[0], exp.shape[1])
    assert same_bits(got, exp)


def test_edge_fixtures_cover_special_scales(dq):
    raw = dq["Q4_K/edge/bytes"]
    d = np.ascontiguousarray(raw[:, 0:2]).view(np.float16).ravel()
    assert np.isnan(d).any() and np.isinf(d).any() and (d == 0).any()
    assert (np.abs(d[np.isfinite(d)]) < 6.2e-5).any()  # subnormal fp16


def test_dequant_shape_errors():
    with pytest.raises(ValueError, match="in_features"):
        ggml_blocks.dequantize(np.zeros(144, np.uint8), "Q4_K", 1, 100)
    with pytest.raises(ValueError, match="does not match"):
        ggml_blocks.dequantize(np.zeros(143, np.uint8), "Q4_K", 1, 256)


@pytest.mark.parametrize("case", ["k4", "k5", "k6"])
def test_mixlinear_matches_reference_autograd(golden_dir, case):
    z = np.load(golden_dir / "mixlinear_golden.npz")
    fmts = list(z[f"{case}/formats"])
    tau = float(z[f"{case}/tau"])
    x, dy, gates = z[f"{case}/x"], z[f"{case}/dy"], z[f"{case}/gates"]
    out_f, in_f = dy.shape[1], x.shape[1]
    cands = mixgemm.decode_candidates([z[f"{case}/cand{k}/bytes"] for k in range(len(fmts))], fmts, out_f, in_f,
                                      in_f)
    p = mixgemm.softmax_probs(gates, tau)
    w = mixgemm.mixed_weight(cands, p)
    assert rel_err(mixgemm.linear_fwd(x, w), z[f"{case}/y"]) < 1e-5
    assert rel_err(mixgemm.linear_dx(dy, w), z[f"{case}/dx"]) < 1e-5
    g = mixgemm.prob_grad(dy, x, cands)
    assert rel_err(g, z[f"{case}/dprobs"]) < 1e-5
    assert rel_err(mixgemm.gate_grad(p, g, tau), z[f"{case}/dgates"]) < 1e-5


@pytest.mark.parametrize("case", ["t1", "t2"])
def test_loss_matches_reference_chunked_loss(golden_dir, case):
    z = np.load(golden_dir / "loss_golden.npz")
    s = z[f"{case}/student"]
    V = s.shape[-1]
    ce, kl, g = oloss.loss_and_grad(s.reshape(-1, V), z[f"{case}/teacher"].reshape(-1, V),
                                    z[f"{case}/targets"].reshape(-1), float(z[f"{case}/temperature"]))
    assert abs(ce - float(z[f"{case}/ce"])) < 1e-5 * abs(float(z[f"{case}/ce"]))
    assert abs(kl - float(z[f"{case}/kl"])) < 1e-5 * abs(float(z[f"{case}/kl"]))
    assert rel_err(g, z[f"{case}/dlogits"].reshape(-1, V)) < 1e-5


def test_assignment_first_max_wins():
    assert mixgemm.assignment(np.array([0.5, 2.0, 2.0, -1.0]), ["a", "b", "c", "d"]) == "b"


def test_ptqr_oracle_matches_reference_routed_functions(golden_dir):
    """The routed forward and its straight-through backward against the
    reference's own _RoutedMixedLinear / _MixedEmbeddingRowFunctionLazy."""
    from oracle import ggml_blocks, mixgemm

    z = np.load(golden_dir / "ptqr_golden.npz")
    fmts = [str(f) for f in z["lin/formats"]]
    y = z["lin/y"]
    OUT, IN = z["lin/dy"].shape[1], z["lin/x"].shape[1]
    cands = [ggml_blocks.dequantize(z[f"lin/cand{k}/bytes"], f, OUT, IN) for k, f in enumerate(fmts)]
    x, dy, routing = z["lin/x"], z["lin/dy"], z["lin/routing"]
    assert np.allclose(mixgemm.routed_linear_fwd(x, cands, routing), y, rtol=1e-4, atol=1e-5)
    probs = mixgemm.softmax_probs(z["lin/gates"], float(z["lin/tau"]))
    w_mix = mixgemm.mixed_weight(cands, probs)
    assert np.allclose(mixgemm.linear_dx(dy, w_mix), z["lin/dx"], rtol=1e-4, atol=1e-5)
    assert np.allclose(mixgemm.prob_grad(dy, x, cands), z["lin/dprobs"], rtol=1e-4, atol=1e-3)
    # embedding rows: exact decode of the routed candidate, rounded once to bf16
    V, D = 64, 512
    rows = z["emb/row_ids"]
    by_cand = [ggml_blocks.dequantize(z[f"emb/cand{k}/bytes"], f, V, D)[rows] for k, f in enumerate(fmts)]
    got = mixgemm.routed_rows(by_cand, z["emb/routing"])
    assert np.array_equal(got.view(np.uint32), z["emb/rows"].astype(np.float32).view(np.uint32))


def test_routing_sampler_shares_follow_probabilities():
    import torch
    from voodoo_quant.layers import _sample_token_routing

    torch.manual_seed(0)
    p = torch.tensor([0.1, 0.6, 0.05, 0.25])
    r = _sample_token_routing(p, 200000)
    shares = torch.bincount(r, minlength=4).double() / r.numel()
    assert torch.allclose(shares, p.double(), atol=5e-3)
