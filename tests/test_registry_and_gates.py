"""Host-side behaviour the reference's own unit tests pin, checked against
this package on CPU (no kernels): the quant-type registry and ladder
(reference tests/test_ggml.py), the gate temperature and per-role candidate
menus (tests/test_invariants.py), and the error conventions of the
boundary."""

from __future__ import annotations

import pytest
import torch

from voodoo_quant import ggml
from oracle import ggml_blocks


def test_registry_ladder_and_sizes():
    types = ggml.list_quant_types()
    assert {"IQ4_XS", "Q8_0", "Q2_K", "Q3_K"} <= set(types)
    ladder = ggml.QUANT_LADDER
    assert set(ladder) <= set(types)
    sizes = [ggml.bytes_per_weight(q) for q in ladder]
    assert sizes == sorted(sizes)  # coarse to fine
    menu = ggml.default_candidate_types()
    assert not any(q.startswith("TQ") for q in menu)
    assert menu[0] == "IQ1_S" and menu[-1] == "Q8_0"
    assert ggml.bytes_per_weight("Q8_0") == pytest.approx(34 / 32)
    assert ggml.bytes_per_weight("IQ4_XS") == pytest.approx(136 / 256)
    assert ggml.bytes_per_weight("Q2_K") == pytest.approx(84 / 256)
    assert ggml.bytes_per_weight("Q3_K") == pytest.approx(110 / 256)
    with pytest.raises(ValueError, match="Unknown quant type"):
        ggml.get_quant_info("NOT_A_TYPE")


def test_gpu_formats_match_the_block_layouts():
    for q in ggml.GPU_FORMATS:
        info = ggml.get_quant_info(q)
        type_id, elems, nbytes = ggml_blocks.FORMATS[q]
        assert (info.block_size, info.block_bytes) == (elems, nbytes), q
        assert info.ggml_type == type_id, q


def test_quantize_without_libggml_is_a_runtime_error():
    if ggml.find_libggml() is not None:
        pytest.skip("libggml-base present")
    with pytest.raises(RuntimeError):
        ggml.quantize_tensor(torch.zeros(4, 256), "Q4_K")


def _layer(types, name="blk.0.mlp.up_proj"):
    from voodoo_quant.layers import MixedQuantLinear
    from voodoo_quant.quants import rtn

    w = torch.randn(32, 256, generator=torch.Generator().manual_seed(1)) * 0.02
    return MixedQuantLinear(256, 32, list(types), w, tensor_name=name,
                            candidate_bytes={q: rtn.quantize(w, q) for q in types})


def test_temperature_concentrates_the_mixture():
    m = _layer(["Q4_K", "Q6_K", "Q8_0"])
    with torch.no_grad():
        m.gates.copy_(torch.tensor([0.1, 0.7, 0.3]))
    m.set_temperature(1.0)
    warm = m.soft_probs()
    m.set_temperature(0.01)
    cold = m.soft_probs()
    assert torch.allclose(warm.sum(), torch.tensor(1.0)) and torch.allclose(cold.sum(), torch.tensor(1.0))
    assert cold.max() > warm.max() and float(cold[1].detach()) > 0.999
    assert m.get_assignment() == "Q6_K"
    m.set_temperature(0.0)  # clamped, never a division by zero
    assert m.temperature > 0 and torch.isfinite(m.soft_probs()).all()
    # effective bytes: the probability-weighted bytes of the full tensor
    eb = float(m.effective_bytes().detach())
    probs = m.soft_probs().detach()
    want = sum(float(p) * ggml.bytes_per_weight(q) for p, q in zip(probs, m.candidate_types)) * 32 * 256
    assert eb == pytest.approx(want, rel=1e-6)


def test_role_menus():
    from voodoo_quant.layers import resolve_candidate_types

    base = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]
    attn, other = ["Q4_K", "Q5_K", "Q6_K", "Q8_0"], ["Q2_K", "Q3_K", "Q4_K"]
    assert resolve_candidate_types("model.layers.0.self_attn.q_proj", base) == base
    assert resolve_candidate_types("model.layers.0.self_attn.q_proj", base, attn, other) == attn
    assert resolve_candidate_types("model.layers.0.mlp.down_proj", base, attn, other) == other
    # a role menu never adds types outside the base menu
    assert resolve_candidate_types("model.layers.0.mlp.up_proj", ["Q4_K", "Q8_0"], attn, other) == ["Q4_K"]


def test_boundary_error_conventions():
    from voodoo_quant.layers import MixedQuantLinear

    w = torch.zeros(32, 256)
    with pytest.raises(ValueError, match="Unknown quant type"):
        MixedQuantLinear(256, 32, ["NOT_A_TYPE"], w)
    with pytest.raises(ValueError, match="no B200 decoder"):
        MixedQuantLinear(256, 32, ["IQ2_XS"], w)
    m = _layer(["Q4_K", "Q8_0"])
    with pytest.raises(RuntimeError):  # no CPU fallback for the gated forward
        m(torch.zeros(2, 256))
    assert issubclass(MixedQuantLinear, torch.nn.Module)


def test_row_chunks_cover_rows_on_256_boundaries():
    from voodoo_quant.layers import _row_chunks

    for T, n in [(600, 3), (8192, 2), (100, 4), (257, 2), (4096, 1)]:
        ch = _row_chunks(T, n)
        assert ch[0][0] == 0 and ch[-1][1] == T
        assert all(a < b for a, b in ch) and all(ch[i][1] == ch[i + 1][0] for i in range(len(ch) - 1))
        assert all(a % 256 == 0 for a, _ in ch) and len(ch) <= max(n, 1)


def test_bank_routing_on_cpu():
    """One batched Gumbel-argmax draw per step for every layer: padding
    candidates are never chosen, each layer's shares follow its
    probabilities, and a second request of the same size reuses the draw."""
    from voodoo_quant.layers import GateBank

    mods = {"a": _layer(["Q4_K", "Q8_0"], "l.a"), "b": _layer(["Q4_K", "Q5_K", "Q6_K", "Q8_0"], "l.b")}
    with torch.no_grad():
        mods["a"].gates.copy_(torch.tensor([0.4, -0.4]))
        mods["b"].gates.copy_(torch.tensor([1.0, 0.0, -1.0, 0.5]))
    bank = GateBank(mods)
    bank.probs()
    torch.manual_seed(0)
    for m in mods.values():
        r = bank.routing(m, 100000).long()
        assert int(r.max()) < m.num_candidates
        shares = torch.bincount(r, minlength=m.num_candidates).double() / r.numel()
        assert torch.allclose(shares, m.get_probs().detach().double(), atol=8e-3)
        assert torch.equal(bank.routing(m, 100000), r.to(torch.uint8))
    bank.release()
    assert mods["a"].__dict__.get("_bank_probs") is None


def test_reference_helpers_kept_for_drop_in():
    """Names the reference's trainer and tools import from layers / parallel
    exist and behave as there (layers.py:225-295, :821-836, :947-960;
    parallel.py:393-408)."""
    from voodoo_quant import layers, parallel
    from voodoo_quant.quants import rtn

    assert layers._format_duration(None) == "..." and layers._format_duration(4.23) == "4.2s"
    assert layers._format_duration(123) == "2m03s" and layers._format_duration(3 * 3600 + 7 * 60) == "3h07m"
    assert layers._quant_info_for("Q4_K").block_bytes == 144
    layers.set_st_gumbel(False, 0.5, 1.0)
    layers.set_st_gumbel_anneal(0.1, 0.9, 100)
    layers.st_gumbel_step(3)
    with pytest.raises(NotImplementedError):
        layers.set_st_gumbel(True, 0.5, 1.0)
    layers.install_heap_dump_handler()
    w = torch.randn(12, 256, generator=torch.Generator().manual_seed(3))
    full = rtn.quantize(w, "Q8_0")
    assert torch.equal(parallel._slice_q8_bytes(full, 12, 256, row_range=(4, 9)), rtn.quantize(w[4:9], "Q8_0"))
    assert torch.equal(parallel._slice_q8_bytes(full, 12, 256, col_range=(64, 192)),
                       rtn.quantize(w[:, 64:192].contiguous(), "Q8_0"))
    idx = torch.tensor([7, 1, 3])
    assert torch.equal(parallel._slice_q8_bytes(full, 12, 256, row_index=idx), rtn.quantize(w[idx], "Q8_0"))
    with pytest.raises(ValueError, match="32-aligned"):
        parallel._slice_q8_bytes(full, 12, 256, col_range=(16, 80))


def test_architecture_adapters():
    from types import SimpleNamespace

    from voodoo_quant.arch import adapter_for_config, adapter_for_gguf_arch

    names = {t: adapter_for_config(SimpleNamespace(model_type=t)).__name__
             for t in ("llama", "qwen3", "qwen3_5", "qwen3_5_text", "lfm2")}
    assert names == {"llama": "LlamaDenseAdapter", "qwen3": "LlamaDenseAdapter", "qwen3_5": "QwenHybridAdapter",
                     "qwen3_5_text": "QwenHybridAdapter", "lfm2": "LFM2Adapter"}
    assert adapter_for_config(SimpleNamespace(model_type="gpt2")) is None
    lfm = adapter_for_gguf_arch("lfm2")
    assert lfm.gguf_name("model.layers.3.conv.in_proj.weight") == "blk.3.shortconv.in_proj.weight"
    assert lfm.gguf_name("model.layers.0.self_attn.out_proj.weight") == "blk.0.attn_output.weight"
    assert lfm.gguf_name("model.layers.5.feed_forward.w3.weight") == "blk.5.ffn_up.weight"
    assert lfm.gguf_name("model.embed_tokens.weight") == "token_embd.weight" and lfm.transpose_embedding()
    assert lfm.gguf_name("lm_head.weight") is None
    assert adapter_for_gguf_arch("qwen35").gguf_name("model.layers.0.mlp.up_proj.weight") is None
    assert adapter_for_gguf_arch("qwen35").is_attention_tensor("model.layers.0.linear_attn.in_proj_qkv.weight")
