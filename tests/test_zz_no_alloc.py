"""vq_gategrad_noalloc: the gate gradient on the library's own fixed scratch,
for callers that cannot allocate device memory.  Called through the C ABI and
checked against vq_gategrad (caller workspace) on the same inputs, on calls
in a row with different shapes and inputs, so that scratch left by one call
cannot pass for the next one's result: the largest shape first, then one
whose tiles outnumber the CTA pairs without dividing by them (its stream-K
tail writes partial slots of its own), then a small single-CTA shape.  Both
entry points run the same deterministic kernels into the same slot layout,
so the results must be bit-identical.  A second round of the same calls
must leave torch's allocation count and the device's free memory unchanged.

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

    g = torch.Generator(device=cuda).manual_seed(seed)
    w = torch.randn(N, IN, generator=g, device=cuda) * 0.02
    blocks = [rtn.quantize(w, q) for q in types]
    x = torch.randn(T, IN, generator=g, device=cuda).to(torch.bfloat16)
    dy = torch.randn(T, N, generator=g, device=cuda).to(torch.bfloat16)
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


def _no_alloc(lib, dy, x, N, IN, types, blocks, out=None):
    K, t, p = _abi_args(types, blocks)
    if out is None:
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
    cases = [
        # (types, T, N, Kin, seed): the largest scratch user first
        (["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 512, 8192, 8192, 23),
        # 16 x 32 = 512 tiles of 256 x 256 over the CTA pairs: a stream-K tail
        (["Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 1000, 4096, 8192, 21),
        # single-CTA shape (N <= 128) with six candidates
        (["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 300, 96, 768, 22),
    ]
    for types, T, N, IN, _ in cases:
        assert lib.vq_gategrad_workspace_bytes(N, IN, len(types)) <= 4 << 20
    inputs = [_inputs(cuda, types, T, N, IN, seed) for types, T, N, IN, seed in cases]
    # the allocation-free calls run back to back; each reuses the scratch the previous one left
    got = [_no_alloc(lib, dy, x, c[2], c[3], c[0], blocks) for c, (x, dy, blocks) in zip(cases, inputs)]
    want = [_with_workspace(lib, dy, x, c[2], c[3], c[0], blocks) for c, (x, dy, blocks) in zip(cases, inputs)]
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    for c, a, b in zip(cases, got, want):
        assert torch.isfinite(a).all()
        assert torch.equal(a, b), (c[0], c[2], c[3], a, b)

    # the same calls again into preallocated outputs: nothing is allocated
    outs = [torch.empty(len(c[0]), dtype=torch.float32, device=cuda) for c in cases]
    torch.cuda.synchronize()
    before = (torch.cuda.memory_allocated(cuda), torch.cuda.mem_get_info(cuda)[0])
    for c, (x, dy, blocks), o in zip(cases, inputs, outs):
        _no_alloc(lib, dy, x, c[2], c[3], c[0], blocks, out=o)
    torch.cuda.synchronize()
    after = (torch.cuda.memory_allocated(cuda), torch.cuda.mem_get_info(cuda)[0])
    assert after == before, (before, after)
    for o, b in zip(outs, want):
        assert torch.equal(o, b)
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
