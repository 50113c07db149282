"""Q8_0 quantiser: the CPU restatement (oracle/q8_quant.py) and the torch
rule of the synthetic packer (quants/rtn.py) against gguf-py's output
(tests/golden/q8quant_golden.npz), byte for byte; the CUDA quantiser
(vq_quantize) is checked against the same vectors in tests/test_gpu_q8_quant.py."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from oracle.q8_quant import quantize_q8_0

GOLDEN = np.load(Path(__file__).parent / "golden" / "q8quant_golden.npz")


def test_oracle_matches_gguf_py():
    with np.errstate(over="ignore"):
        assert np.array_equal(quantize_q8_0(GOLDEN["w"]), GOLDEN["q"])
        assert np.array_equal(quantize_q8_0(GOLDEN["w_bf16"]), GOLDEN["q_bf16"])


def test_ties_round_half_away_from_zero():
    q = GOLDEN["q"].reshape(24, 8, 34)[1, 0, 2:].view(np.int8)
    assert q[:8].tolist() == [127, 1, 2, 3, -1, -2, -3, 0]  # 0.49999997 -> 0
    assert q[9:11].tolist() == [127, -127]


def test_synthetic_packer_matches_gguf_py():
    from voodoo_quant.quants import rtn

    got = rtn.quantize(torch.from_numpy(GOLDEN["w"]), "Q8_0").numpy()
    assert np.array_equal(got, GOLDEN["q"])
