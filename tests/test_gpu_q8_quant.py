"""CUDA Q8_0 quantiser (vq_quantize) against gguf-py's bytes
(tests/golden/q8quant_golden.npz) and the CPU restatement (oracle/q8_quant.py):
byte-exact, from float32 and bfloat16 weights, strided rows, and the
errors of the boundary."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.q8_quant import quantize_q8_0

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).parent / "golden" / "q8quant_golden.npz")


def test_golden_bytes(cuda):
    from voodoo_quant import _C

    w = torch.from_numpy(GOLDEN["w"]).to(cuda)
    assert np.array_equal(_C.quantize(w, "Q8_0").cpu().numpy(), GOLDEN["q"])
    wb = torch.from_numpy(GOLDEN["w_bf16"]).to(cuda).to(torch.bfloat16)
    assert np.array_equal(_C.quantize(wb, "Q8_0").cpu().numpy(), GOLDEN["q_bf16"])
    assert _C.device_error() == 0


def test_large_and_strided_match_oracle(cuda):
    from voodoo_quant import _C

    g = torch.Generator().manual_seed(3)
    w = torch.randn(4096, 4096 + 64, generator=g) * torch.exp(torch.randn(4096, 1, generator=g))
    view = w[:, 32:32 + 4096]  # leading dimension 4160, 128-byte offset
    got = _C.quantize(view.to(cuda), "Q8_0").cpu().numpy()
    assert np.array_equal(got, quantize_q8_0(view.contiguous().numpy()))
    full = _C.quantize(w.to(cuda)[:, 32:32 + 4096], "Q8_0").cpu().numpy()  # strided device view
    assert np.array_equal(full, got)


def test_boundary_errors(cuda):
    from voodoo_quant import _C

    with pytest.raises(ValueError):
        _C.quantize(torch.zeros(4, 256, device=cuda), "Q4_K")  # GPU quantiser is Q8_0 only
    with pytest.raises(ValueError):
        _C.quantize(torch.zeros(4, 48, device=cuda), "Q8_0")  # cols % 32
    assert _C.quantize(torch.zeros(0, 64, device=cuda), "Q8_0").shape == (0, 34)


def test_quantize_tensor_uses_the_gpu_for_q8_0(cuda):
    from voodoo_quant.ggml import quantize_tensor

    w = torch.from_numpy(GOLDEN["w"]).to(cuda)
    q = quantize_tensor(w, "Q8_0")
    assert q.is_cuda and np.array_equal(q.cpu().numpy(), GOLDEN["q"])
