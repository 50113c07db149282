"""vq_gategrad_noalloc: the gate gradient on the library's own fixed scratch,
for callers that cannot allocate device memory.  Called through the C ABI and
checked against vq_gategrad (caller workspace) on the same inputs, on two
calls in a row with different inputs, so that scratch left by the first call
cannot pass for the second's result.  Tolerance: the gate-gradient tolerance
of the kernel tests, 1e-3 relative.

This file is collected last on purpose: it must pass alone in a fresh process
and after every other test has run in the same process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import rel_err


def _inputs(cuda, types, T, N, IN, seed):
    from voodoo_quant.quants import rtn

    g = torch.Generator(device="cpu").manual_seed(seed)
    w = torch.randn(N, IN, generator=g) * 0.02
    blocks = [rtn.quantize(w, q).to(cuda) for q in types]
    x = torch.randn(T, IN, generator=g).to(cuda, torch.bfloat16)
    dy = torch.randn(T, N, generator=g).to(cuda, torch.bfloat16)
    return x, dy, blocks


def _abi_args(types, blocks):
    from voodoo_quant import _C

    K = len(types)
    t = (ctypes.c_int * K)(*[_C.GGML_TYPE[q] for q in types])
    p = (ctypes.c_void_p * K)(*[b.data_ptr() for b in blocks])
    return K, t, p


def _with_workspace(lib, dy, x, N, IN, types, blocks):
    K, t, p = _abi_args(types, blocks)
    need = lib.vq_gategrad_workspace_bytes(N, IN, K)
    ws = torch.empty(need, dtype=torch.uint8, device=x.device)
    out = torch.empty(K, dtype=torch.float32, device=x.device)
    st = torch.cuda.current_stream(x.device).cuda_stream
    rc = lib.vq_gategrad(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), x.shape[0], N, IN, K, t, p, IN,
                         ws.data_ptr(), ws.numel(), out.data_ptr(), st)
    assert rc == 0, lib.vq_last_error()
    return out


def _no_alloc(lib, dy, x, N, IN, types, blocks):
    K, t, p = _abi_args(types, blocks)
    out = torch.empty(K, dtype=torch.float32, device=x.device)
    st = torch.cuda.current_stream(x.device).cuda_stream
    rc = lib.vq_gategrad_noalloc(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), x.shape[0], N, IN, K, t, p,
                                 IN, out.data_ptr(), st)
    assert rc == 0, lib.vq_last_error()
    return out


@pytest.mark.gpu
def test_no_alloc_gategrad_matches_workspace_entry_point(cuda):
    from voodoo_quant import _C

    lib = _C.load_library()
    # a paired-CTA shape (N > 128) with five candidates, then a single-CTA shape with six
    cases = [(["Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 1000, 1536, 2048, 21),
             (["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 300, 96, 768, 22)]
    inputs = [_inputs(cuda, types, T, N, IN, seed) for types, T, N, IN, seed in cases]
    # the two allocation-free calls run back to back; the second reuses the scratch the first left
    got = [_no_alloc(lib, dy, x, c[2], c[3], c[0], blocks) for c, (x, dy, blocks) in zip(cases, inputs)]
    want = [_with_workspace(lib, dy, x, c[2], c[3], c[0], blocks) for c, (x, dy, blocks) in zip(cases, inputs)]
    torch.cuda.synchronize()
    for c, a, b in zip(cases, got, want):
        assert torch.isfinite(a).all()
        assert rel_err(a.cpu().numpy(), b.cpu().numpy()) < 1e-3, (c[0], a, b)
    assert _C.device_error() == 0


def test_no_alloc_gategrad_rejects_oversized_layers():
    """The size check comes before any CUDA call, so it runs without a GPU."""
    from voodoo_quant import _C

    lib = _C.load_library()
    limit = 4 << 20
    N, IN, K = 262144, 8192, 8
    assert lib.vq_gategrad_workspace_bytes(N, IN, K) > limit
    types = (ctypes.c_int * K)(*([_C.GGML_TYPE["Q8_0"]] * K))
    ptrs = (ctypes.c_void_p * K)(*([None] * K))
    rc = lib.vq_gategrad_noalloc(None, IN, None, IN, 16, N, IN, K, types, ptrs, IN, None, None)
    assert rc == _C.VQ_ERR_INVALID
    assert b"scratch" in lib.vq_last_error()
    # the largest vocabulary projection of the benchmark shapes fits
    assert lib.vq_gategrad_workspace_bytes(152064, 5120, 7) <= limit
