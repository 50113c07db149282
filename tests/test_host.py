"""Host-side logic that needs no GPU: the C-ABI library's exports, the
round-to-nearest block packer, the candidate cache format and the module API."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import ROOT
from oracle import ggml_blocks

HEADER = ROOT / "include" / "voodoo_b200.h"


def _declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?(?:int|size_t|char\s*\*|const char\s*\*)\s*\*?\s*(vq_\w+)\s*\(",
                                 text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from voodoo_quant import _C

    lib = _C.load_library()
    syms = _declared_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_C.EXPORTED)
    assert lib.vq_abi_version() == 1


def test_library_validation_paths_without_gpu():
    from voodoo_quant import _C

    lib = _C.load_library()
    be, bb = ctypes.c_int(), ctypes.c_int()
    assert lib.vq_format_info(12, ctypes.byref(be), ctypes.byref(bb)) == 0 and (be.value, bb.value) == (256, 144)
    assert lib.vq_format_info(8, ctypes.byref(be), ctypes.byref(bb)) == 0 and (be.value, bb.value) == (32, 34)
    assert lib.vq_format_info(999, None, None) == _C.VQ_ERR_UNSUPPORTED
    assert b"unsupported" in lib.vq_last_error()
    # shape validation happens before any CUDA call
    assert lib.vq_dequant(12, None, 4, 100, None, None) == _C.VQ_ERR_INVALID
    assert lib.vq_dequant(12, None, 0, 256, None, None) == 0  # empty input is a no-op
    # the mixture conveniences validate their candidates before any launch
    for fn in (lib.vq_mixgemm_fwd, lib.vq_mixgemm_dx):
        assert fn(None, 8, 8, 8, 0, None, None, None, 8, 256, None, 256, None, 8, None) == _C.VQ_ERR_INVALID
        assert b"candidates" in lib.vq_last_error()
    # per-tile slots (112 row blocks x 16 column blocks x 4 warps) + 16 stream-K slots per CTA pair (<= 128)
    assert lib.vq_gategrad_workspace_bytes(14336, 4096, 5) == (112 * 16 * 4 + 16 * 128) * 5 * 4


@pytest.mark.parametrize("fmt,ceiling", [("Q8_0", 0.02), ("Q6_K", 0.05), ("Q5_K", 0.08), ("Q4_K", 0.12),
                                         ("IQ4_XS", 0.12), ("Q3_K", 0.25), ("Q2_K", 0.45)])
def test_rtn_packer_round_trip(fmt, ceiling):
    """Error ceilings in the style of the reference's tests/test_ggml.py:37-49."""
    from voodoo_quant.quants import rtn

    torch.manual_seed(0)
    w = torch.randn(8, 512)
    qb = rtn.quantize(w, fmt)
    _, bs, bb = ggml_blocks.FORMATS[fmt]
    assert qb.dtype == torch.uint8 and qb.shape == (8 * 512 // bs, bb)
    deq = ggml_blocks.dequantize(qb.numpy(), fmt, 8, 512)
    err = np.abs(deq - w.numpy()).mean() / np.abs(w.numpy()).mean()
    assert err < ceiling


def test_rtn_q8_0_matches_ggml_reference_rule():
    """Q8_0 packing is ggml's reference rule; gguf-py implements it bit-exactly."""
    gguf = pytest.importorskip("gguf")
    from gguf import quants as gq
    from voodoo_quant.quants import rtn

    torch.manual_seed(1)
    w = torch.randn(4, 256) * 0.05
    ours = rtn.quantize(w, "Q8_0").numpy().reshape(-1)
    ref = gq.quantize(w.numpy(), gguf.GGMLQuantizationType.Q8_0).reshape(-1)
    assert np.array_equal(ours, ref)


def test_registry_has_benchmark_formats():
    from voodoo_quant import ggml

    for name, (tid, bs, bb) in ggml_blocks.FORMATS.items():
        info = ggml.get_quant_info(name)
        assert (info.ggml_type, info.block_size, info.block_bytes) == (tid, bs, bb)
    with pytest.raises(ValueError, match="Unknown quant type"):
        ggml.get_quant_info("Q7_K")
    assert ggml.get_quant_info("Q4_K").quant_func == "quantize_q4_K"


def _module(types=("Q4_K", "Q8_0"), out_f=64, in_f=512, **kw):
    from voodoo_quant.layers import MixedQuantLinear
    from voodoo_quant.quants import rtn

    torch.manual_seed(0)
    w = torch.randn(out_f, in_f) * 0.02
    cb = {q: rtn.quantize(w, q) for q in types}
    return MixedQuantLinear(in_f, out_f, list(types), w, candidate_bytes=cb, tensor_name="t.w", **kw), w, cb


def test_module_api_and_budget():
    from voodoo_quant import ggml

    m, w, cb = _module()
    assert m.num_candidates == 2 and m.padded_in_features == 512
    assert torch.equal(m._qweight_0.cpu(), cb["Q4_K"]) and torch.equal(m._qweight_1.cpu(), cb["Q8_0"])
    eb = m.effective_bytes().item()
    expect = 0.5 * (ggml.bytes_per_weight("Q4_K") + ggml.bytes_per_weight("Q8_0")) * 64 * 512
    assert abs(eb - expect) < 1e-3 * expect
    with torch.no_grad():
        m.gates.copy_(torch.tensor([1.0, 1.0]))
    assert m.get_assignment() == "Q4_K"  # first maximum wins, like torch.argmax
    m.set_temperature(0.0)
    assert m.temperature == 1e-6


def test_unsupported_candidate_rejected():
    with pytest.raises(ValueError):
        _module(types=("IQ2_XXS",))
    with pytest.raises(ValueError):
        _module(types=("Q9_Z",))


def test_candidate_cache_format_round_trip(tmp_path, monkeypatch):
    """A combined_lazy cache file in the reference's format is found and used."""
    from voodoo_quant import layers
    from voodoo_quant.quants import rtn

    monkeypatch.setattr(layers, "_CANDIDATE_CACHE_ROOT", tmp_path)
    torch.manual_seed(0)
    w = torch.randn(32, 300)  # in_features padded to 512
    padded, _, _ = layers._pad_weight_and_imatrix(w, None)
    cb = {q: rtn.quantize(padded, q) for q in ("Q5_K", "Q6_K")}
    path = layers._combined_cache_path("model.layers.0.mlp.up_proj", "lazy", layers._tensor_hash(w), "none")
    torch.save(cb, path)
    assert path.name.startswith("combined_lazy_w") and path.parent.name == "model_layers_0_mlp_up_proj"
    m = layers.MixedQuantLinear(300, 32, ["Q5_K", "Q6_K"], w, tensor_name="model.layers.0.mlp.up_proj")
    assert m.padded_in_features == 512
    assert torch.equal(m._qweight_1.cpu(), cb["Q6_K"])
    # the alternate `model.`-less name is also accepted (reference layers.py:1116-1121)
    m2 = layers.MixedQuantLinear(300, 32, ["Q5_K"], w, tensor_name="layers.0.mlp.up_proj")
    assert torch.equal(m2._qweight_0.cpu(), cb["Q5_K"])


def test_missing_candidates_are_quantized_on_threads_and_cached(tmp_path, monkeypatch):
    """Cache-cold candidates are quantized concurrently (one thread each, as
    the reference's _quantize_candidates_parallel) and saved to the cache;
    a second layer over the same weight then loads them without quantizing."""
    import threading
    import time

    from voodoo_quant import layers
    from voodoo_quant.quants import rtn

    monkeypatch.setattr(layers, "_CANDIDATE_CACHE_ROOT", tmp_path)
    types = ["Q4_K", "Q5_K", "Q6_K", "Q8_0"]
    calls, threads = [], set()

    def fake_quantize(w, qt, im=None):  # stands in for libggml's quantize_* (which runs outside the GIL)
        calls.append(qt)
        threads.add(threading.get_ident())
        time.sleep(0.3)
        return rtn.quantize(w, qt)

    monkeypatch.setattr(layers, "quantize_tensor", fake_quantize)
    monkeypatch.setenv("VOODOO_QUANT_WORKERS", "4")
    w = torch.randn(16, 256) * 0.02
    t0 = time.perf_counter()
    m = layers.MixedQuantLinear(256, 16, types, w, tensor_name="cold.proj")
    assert time.perf_counter() - t0 < 1.0  # four 0.3 s quantizations side by side, not 1.2 s in a row
    assert sorted(calls) == sorted(types) and len(threads) == 4
    for k, qt in enumerate(types):
        assert torch.equal(getattr(m, f"_qweight_{k}").cpu(), rtn.quantize(w, qt))
    calls.clear()
    layers.MixedQuantLinear(256, 16, types, w, tensor_name="cold.proj")
    assert calls == []  # served from the cache files written above


def test_missing_candidates_need_libggml(tmp_path, monkeypatch):
    from voodoo_quant import ggml, layers

    monkeypatch.setattr(layers, "_CANDIDATE_CACHE_ROOT", tmp_path)
    monkeypatch.setattr(ggml, "find_libggml", lambda: None)
    monkeypatch.setattr(ggml, "_LIB", None)
    with pytest.raises(RuntimeError, match="libggml-base.so not found"):
        layers.MixedQuantLinear(256, 8, ["Q4_K"], torch.randn(8, 256), tensor_name="nope")


def test_shard_rows_and_cols_slice_packed_blocks():
    m, w, cb = _module(types=("Q4_K", "Q8_0"), out_f=64, in_f=1024)
    m.shard_rows([(8, 24), (40, 48)])
    assert m.out_features == 24 and m._full_out_features == 64
    q4 = cb["Q4_K"].reshape(64, 4, 144)
    assert torch.equal(m._qweight_0.cpu().reshape(24, 4, 144), torch.cat([q4[8:24], q4[40:48]]))
    with pytest.raises(RuntimeError, match="already"):
        m.shard_cols((0, 256))
    m2, _, cb2 = _module(types=("Q4_K", "Q8_0"), out_f=16, in_f=1024)
    m2.shard_cols((256, 768))
    assert m2.in_features == 512 and m2.padded_in_features == 512
    q8 = cb2["Q8_0"].reshape(16, 32, 34)
    assert torch.equal(m2._qweight_1.cpu().reshape(16, 16, 34), q8[:, 8:24])
    m3, _, _ = _module(types=("Q4_K",), out_f=16, in_f=1024)
    with pytest.raises(ValueError, match="aligned"):
        m3.shard_cols((128, 512))


def test_resolve_candidate_types_per_role():
    from voodoo_quant.layers import resolve_candidate_types

    base = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]
    assert resolve_candidate_types("model.layers.0.self_attn.q_proj", base, ["Q4_K", "Q5_K", "Q9"], ["Q2_K"]) == \
        ["Q4_K", "Q5_K"]
    assert resolve_candidate_types("model.layers.0.mlp.up_proj", base, ["Q4_K"], ["Q2_K", "Q3_K"]) == ["Q2_K", "Q3_K"]
    assert resolve_candidate_types("x", base) == base


def test_forward_refuses_cpu_tensors():
    m, w, _ = _module()
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(4, 512))


def test_store_accounting():
    from voodoo_quant.cache import STORE

    m, _, cb = _module(types=("Q4_K", "Q6_K"), out_f=32, in_f=512)
    assert STORE.get("t.w") is m
    assert sum(l.nbytes for l in m._cand_layout) == sum(v.numel() for v in cb.values())
    assert all(l.offset % 256 == 0 for l in m._cand_layout)


def test_gate_bank_matches_per_layer_probabilities_and_bytes():
    """The batched per-step gate softmax equals each layer's own, and so do the
    size term and its gradient."""
    from voodoo_quant.layers import GateBank, total_effective_bytes

    mods = {}
    for i, (types, out_f, in_f) in enumerate([(("Q4_K", "Q8_0"), 32, 512), (("Q3_K", "Q4_K", "Q5_K", "Q6_K"), 16, 256),
                                               (("Q6_K",), 8, 256)]):
        m, _, _ = _module(types=types, out_f=out_f, in_f=in_f)
        with torch.no_grad():
            m.gates.copy_(torch.randn(len(types), generator=torch.Generator().manual_seed(i)))
        m.set_temperature(0.3 + i)
        mods[f"l{i}"] = m
    ref_p = [m.soft_probs().detach() for m in mods.values()]
    ref_b = total_effective_bytes(mods)
    ref_b.backward()
    ref_g = [m.gates.grad.clone() for m in mods.values()]
    for m in mods.values():
        m.gates.grad = None
    bank = GateBank(mods)
    bank.probs()
    for m, p in zip(mods.values(), ref_p):
        assert torch.allclose(m.get_probs(), p, rtol=1e-6, atol=1e-7)
    b = bank.effective_bytes()
    assert torch.allclose(b, ref_b, rtol=1e-6)
    b.backward()
    for m, g in zip(mods.values(), ref_g):
        assert torch.allclose(m.gates.grad, g, rtol=1e-4, atol=1e-6)
    bank.release()
    assert all(m.__dict__.get("_bank_probs") is None for m in mods.values())


def test_step_flops_per_token_roofline_denominators():
    """The algorithmic FLOPs per token behind the full-step roofline: 6 x the
    student's gated linear weights (forward, dX, gate-grad GEMM), 4 x a tied
    unquantised head, 2 x the teacher's, causal attention 4 L (S/2) d x 4."""
    import bench
    from voodoo_quant.training import synthetic as S

    def by_hand(L, H, q, kv, hd, F, V, S_, tied):
        p = L * (H * (q + 2 * kv) * hd + q * hd * H + 3 * H * F)
        return 6 * p + (4 if tied else 6) * V * H + 2 * (p + V * H) + 16 * L * (S_ / 2) * q * hd

    assert bench.step_flops_per_token(S.SHAPES["8b"]) == by_hand(32, 4096, 32, 8, 128, 14336, 128256, 4096, False)
    assert bench.step_flops_per_token(S.SHAPES["0.6b"]) == by_hand(28, 1024, 16, 8, 128, 3072, 151936, 2048, True)
    assert bench.step_flops_per_token(S.SHAPES["32b"]) == by_hand(64, 5120, 40, 8, 128, 25600, 152064, 8192, False)
    assert abs(bench.step_flops_per_token(S.SHAPES["8b"]) / 1e9 - 64.33) < 0.01


def test_reference_arm_prints_one_contract_line():
    """bench.py --impl reference (the reference's algorithm on the host) prints
    one JSON line with the keys the benchmark contract names, the GPU arm's
    config object for the same workload, and a ms_per_step it timed."""
    import json
    import subprocess
    import sys
    from pathlib import Path

    import bench
    from voodoo_quant.training import synthetic as S

    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "tiny", "--steps", "2",
                        "--warmup", "1", "--cpu-tokens", "64"], cwd=root, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    out = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in out, key
    assert out["impl"] == "reference" and out["value"] > 0 and out["unit"] == "tokens/s"
    assert out["metric"] == bench.METRIC
    assert out["cpu_baseline"]["kind"] == "port" and out["cpu_baseline"]["cores"] >= 1
    assert out["e2e"]["h2d_bytes_per_step"] == 0
    assert out["config"] == json.loads(json.dumps(bench.step_config("tiny", S.SHAPES["tiny"], 1)))
    assert 0 < out["ms_per_step"] < 60e3


def test_full_step_host_baseline_scales_the_layer_sample():
    """The full-step host baseline: one decoder layer's seven gated Linears
    timed on the host, per-weight time scaled by the student's gated weights
    over the layer's, per-token time by the step's FLOPs over the sample's."""
    import bench
    from voodoo_quant.training import synthetic as S

    shape = S.SHAPES["tiny"]
    s = bench.HostLayerSample(shape, 32)
    roles = [r for r, *_ in s.tensors]
    assert roles == ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]
    assert s.p_layer == 256 * 256 * 4 + 3 * 256 * 768
    assert bench.gated_linear_params(shape) == 2 * s.p_layer + 4096 * 256
    w, t = s.step()
    assert w > 0 and t > 0
    full = s.full_step_s(w, t)
    fpt = bench.step_flops_per_token(shape)
    want = w * bench.gated_linear_params(shape) / s.p_layer + t * fpt * 256 / (6.0 * s.p_layer * 32)
    assert abs(full - want) <= 1e-9 * want
    r = bench.step_cpu_baseline(shape, tokens=32, repeats=1)
    assert r["kind"] == "port" and r["unit"] == "tokens/s" and r["cores"] >= 1 and r["value"] > 0
    assert abs(r["value"] - 256 / r["full_step_s_estimate"]) <= 0.05 * r["value"] + 1e-3
    assert "GFLOP/token" in r["sample"]
