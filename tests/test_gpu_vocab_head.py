"""A gated vocabulary-scale head (the 8B shape's lm_head, 128256 x 4096, K = 6
candidates Q2_K ... Q8_0) through MixedQuantLinear on the B200 kernels.

The reference routes heads this large through ``_BlockedCandidateLinear``
(voodoo_quant/layers.py:1560-1637): y = sum_k p_k X W_k^T in row blocks,
dX = sum_k p_k dY W_k, g_k = <dY^T X, W_k>.  Here the same head runs the
uniform mixture path (one W_mix, one GEMM each way, the gate-gradient GEMM);
the sums are the same mathematics.

Checks: Y on 64 sampled output columns against the CPU oracle (candidate
rows decoded by oracle.ggml_blocks, mixed in float64); dX and the K gate
gradients against a float32 torch reference built from the exact decodes
(_C.dequant, bit-exact to the oracle elsewhere).  Tolerances: Y and dX within
1e-2 relative; the gates' gradient (a K-vector) cosine >= 0.999 and
relative error <= 1e-2.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cosine, rel_err
from oracle import ggml_blocks

pytestmark = pytest.mark.gpu

TYPES = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]


def test_vocab_scale_gated_head_matches_references(cuda):
    from voodoo_quant import _C
    from voodoo_quant.layers import MixedQuantLinear
    from voodoo_quant.quants import rtn

    V, H, T = 128256, 4096, 256
    g = torch.Generator(device=cuda).manual_seed(31)
    w = torch.randn(V, H, generator=g, device=cuda) * 0.02
    head = MixedQuantLinear(H, V, TYPES, w, tensor_name="lm_head",
                            candidate_bytes={q: rtn.quantize(w, q) for q in TYPES})
    del w
    with torch.no_grad():
        head.gates.copy_(torch.randn(len(TYPES), generator=g, device=cuda))
    head.set_temperature(0.8)
    x = torch.randn(T, H, generator=g, device=cuda).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(T, V, generator=g, device=cuda).to(torch.bfloat16)
    probs = head.get_probs().detach()

    y = head(x)
    y.backward(dy)
    torch.cuda.synchronize()
    assert _C.device_error() == 0

    # Y on sampled columns against the CPU oracle
    blocks = head._candidate_blocks()
    cols = torch.randperm(V, generator=torch.Generator().manual_seed(32))[:64].sort().values
    p64 = probs.double().cpu().numpy()
    wmix = np.zeros((64, H))
    for k, (qt, qb) in enumerate(zip(TYPES, blocks)):
        rows = qb.view(V, -1).index_select(0, cols.to(cuda)).cpu().numpy()
        wmix += p64[k] * ggml_blocks.dequantize(rows.reshape(-1), qt, 64, H).astype(np.float64)
    y_ref = x.detach().double().cpu().numpy() @ wmix.T
    assert rel_err(y.detach()[:, cols.to(cuda)].float().cpu().numpy(), y_ref) < 1e-2

    # dX and the gate gradients against float32 torch on the exact decodes
    dyf, xf = dy.float(), x.detach().float()
    dx_ref = torch.zeros(T, H, device=cuda)
    g_ref = np.zeros(len(TYPES))
    for k, (qt, qb) in enumerate(zip(TYPES, blocks)):
        wk = _C.dequant(qb, qt, V, H)
        dx_ref += probs[k] * (dyf @ wk)
        for r0 in range(0, V, 16384):  # <dY^T X, W_k> over row blocks, float64 sums
            dw = dyf[:, r0:r0 + 16384].t() @ xf
            g_ref[k] += float((dw.double() * wk[r0:r0 + 16384].double()).sum())
        del wk
    assert rel_err(x.grad.float().cpu().numpy(), dx_ref.cpu().numpy()) < 1e-2
    # gates.grad = (diag p - p p^T) g / tau; compare g itself through the same Jacobian
    p = probs.double().cpu().numpy()
    gates_ref = p * (g_ref - p @ g_ref) / 0.8
    got = head.gates.grad.double().cpu().numpy()
    assert cosine(got, gates_ref) >= 0.999
    assert rel_err(got, gates_ref) <= 1e-2
