"""Tensor-parallel host logic on CPU: gloo process groups of world size 2.

Covers the pieces of voodoo_quant.parallel that need no GPU: block-aligned
(uneven) splits, packed-block slicing invariants, the differentiable
all-reduce, the exact input-gradient ("f") operator and the flat gate-gradient
all-reduce.  The multi-block gradient test reproduces the reference's TP gate
gradient error (column-parallel layers without an input all-reduce) and shows
the f operator removes it.
"""

from __future__ import annotations

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_block_aligned_split_uneven():
    from voodoo_quant.parallel import block_aligned_split

    parts = [block_aligned_split(25600, 8, r) for r in range(8)]
    assert [n // 256 for _, n in parts] == [13, 13, 13, 13, 12, 12, 12, 12]
    assert parts[0][0] == 0 and all(parts[i][0] + parts[i][1] == parts[i + 1][0] for i in range(7))
    assert sum(n for _, n in parts) == 25600
    assert [n // 256 for _, n in (block_aligned_split(5120, 8, r) for r in range(8))] == [3, 3, 3, 3, 2, 2, 2, 2]
    with pytest.raises(ValueError):
        block_aligned_split(1000, 2, 0)
    with pytest.raises(ValueError):
        block_aligned_split(512, 4, 0)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q8_0", "Q6_K", "Q3_K", "IQ4_XS"])
def test_slice_qbytes_equals_quantizing_the_slice(fmt):
    """Row and 256-aligned column slices of packed blocks equal packing the
    slice (block-local formats), the invariant of the reference's
    tests/test_invariants.py:21-53."""
    from voodoo_quant.parallel import ShardSpec
    from voodoo_quant.quants import rtn

    torch.manual_seed(0)
    w = torch.randn(48, 1024) * 0.02
    full = rtn.quantize(w, fmt)
    rs = ShardSpec(full_out=48, full_in=1024, row_offset=16, row_len=20)
    assert torch.equal(rs.slice_qbytes(full, fmt, 1024), rtn.quantize(w[16:36], fmt))
    cs = ShardSpec(full_out=48, full_in=1024, col_offset=256, col_len=512)
    assert torch.equal(cs.slice_qbytes(full, fmt, 1024).reshape(-1), rtn.quantize(w[:, 256:768], fmt).reshape(-1))
    bad = ShardSpec(full_out=48, full_in=1024, col_offset=128, col_len=256)
    with pytest.raises(ValueError, match="aligned"):
        bad.slice_qbytes(full, fmt, 1024)


def _blocks(torch_mod, d, h):
    g = torch.Generator().manual_seed(7)
    mk = lambda o, i: torch_mod.nn.Linear(i, o, bias=False).double()
    blocks = []
    for _ in range(2):
        b = torch.nn.Module()
        b.mlp = torch.nn.Module()
        b.mlp.gate_proj = mk(h, d)
        b.mlp.up_proj = mk(h, d)
        b.mlp.down_proj = mk(d, h)
        for lin in (b.mlp.gate_proj, b.mlp.up_proj, b.mlp.down_proj):
            with torch.no_grad():
                lin.weight.copy_(torch.randn(lin.weight.shape, generator=g, dtype=torch.float64) * 0.1)
        blocks.append(b)
    return blocks


def _mlp_forward(mlp, x, gate):
    return mlp.down_proj(torch.nn.functional.silu(mlp.gate_proj(x) * gate) * mlp.up_proj(x))


class _MLP(torch.nn.Module):
    def __init__(self, inner, gate):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = inner.gate_proj, inner.up_proj, inner.down_proj
        self.g = gate

    def forward(self, x):
        return _mlp_forward(self, x, self.g)


def _worker(rank, world, port, outdir, exact):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from voodoo_quant import parallel as P

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        P.adopt_process_group(0)
        P.TP.exact_input_grad = exact
        d, h, T = 256, 512, 6
        torch.manual_seed(3)
        x = torch.randn(T, d, dtype=torch.float64)
        gy = torch.randn(T, d, dtype=torch.float64)
        blocks = _blocks(torch, d, h)
        gates = [torch.tensor(1.3, dtype=torch.float64, requires_grad=True) for _ in blocks]
        mlps = [_MLP(b.mlp, g) for b, g in zip(blocks, gates)]
        for m in mlps:
            P.tp_mlp(m)
        hcur = x.clone().requires_grad_(True)
        out = hcur
        for m in mlps:
            out = out + m(out)
        (out * gy).sum().backward()
        # rank-local gate grads are partial sums over this rank's slice; the
        # trainer sums them across ranks (one flat all-reduce here)
        P.all_reduce_gate_grads(gates)
        res = {"gates": [g.grad.item() for g in gates], "dx": hcur.grad.clone(), "y": out.detach().clone()}
        # differentiable all-reduce: forward sums, backward is the identity
        t = torch.full((3,), float(rank + 1), requires_grad=True)
        s = P.tp_all_reduce_sum(t)
        s.sum().backward()
        res["ar"] = s.detach().tolist()
        res["ar_grad"] = t.grad.tolist()
        u = torch.full((4,), float(10 * (rank + 1)))
        P.tp_all_reduce_async(u).wait()
        res["ar_async"] = u.tolist()
        torch.save(res, os.path.join(outdir, f"r{rank}_{int(exact)}.pt"))
    finally:
        P.reset_tp()
        dist.destroy_process_group()


def _reference(d=256, h=512, T=6):
    torch.manual_seed(3)
    x = torch.randn(T, d, dtype=torch.float64)
    gy = torch.randn(T, d, dtype=torch.float64)
    blocks = _blocks(torch, d, h)
    gates = [torch.tensor(1.3, dtype=torch.float64, requires_grad=True) for _ in blocks]
    hcur = x.clone().requires_grad_(True)
    out = hcur
    for b, g in zip(blocks, gates):
        out = out + _mlp_forward(b.mlp, out, g)
    (out * gy).sum().backward()
    return [g.grad.item() for g in gates], hcur.grad, out.detach()


@pytest.mark.parametrize("exact", [True, False])
def test_tp2_mlp_stack_gate_gradients(exact):
    port = _free_port()
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_worker, args=(2, port, td, exact), nprocs=2, join=True, start_method="spawn")
        r0 = torch.load(os.path.join(td, f"r0_{int(exact)}.pt"))
        r1 = torch.load(os.path.join(td, f"r1_{int(exact)}.pt"))
    g_ref, dx_ref, y_ref = _reference()
    assert torch.allclose(r0["y"], y_ref, rtol=1e-12, atol=1e-12)
    assert r0["gates"] == r1["gates"]
    assert r0["ar"] == [3.0, 3.0, 3.0] and r0["ar_grad"] == [1.0, 1.0, 1.0]
    assert r0["ar_async"] == r1["ar_async"] == [30.0] * 4
    if exact:
        # exact input gradients: the summed gate gradients equal the unsharded ones
        for got, ref in zip(r0["gates"], g_ref):
            assert abs(got - ref) <= 1e-9 * max(1.0, abs(ref))
        assert torch.allclose(r0["dx"], dx_ref, rtol=1e-10, atol=1e-10)
    else:
        # the reference's behaviour: block 1's gate gradient is computed from a
        # partial upstream gradient and is off after the cross-rank sum
        assert abs(r0["gates"][0] - g_ref[0]) > 1e-3 * abs(g_ref[0])


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=1000, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, rms_norm_eps=1e-6,
                      rope_theta=1e4, tie_word_embeddings=False, max_position_embeddings=64)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(11)
    m = LlamaForCausalLM(cfg).double()
    with torch.no_grad():
        for n, p in m.named_parameters():
            p.copy_(torch.randn_like(p) * (0.3 if n.endswith("norm.weight") else 0.05)
                    + (1.0 if n.endswith("norm.weight") else 0.0))
    ids = torch.randint(0, 1000, (2, 12), generator=torch.Generator().manual_seed(2))
    G = torch.randn(2, 12, 1000, dtype=torch.float64, generator=torch.Generator().manual_seed(4))
    return m, ids, G


def _model_worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from voodoo_quant import parallel as P

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        P.adopt_process_group(0)
        m, ids, G = _tiny_llama()
        P.tp_patch_model(m, verbose=False)
        v0, v1 = m.lm_head.tp_vocab_start, m.lm_head.tp_vocab_end
        logits = m(input_ids=ids).logits
        (logits * G[..., v0:v1]).sum().backward()
        norms = {n: p.grad.clone() for n, p in m.named_parameters() if n.endswith("norm.weight")}
        emb = m.model.embed_tokens
        torch.save({"logits": logits.detach(), "v": (v0, v1), "norms": norms,
                    "emb_rows": (emb.tp_vocab_start, emb.tp_vocab_end), "emb_grad": emb.weight.grad.clone()},
                   os.path.join(outdir, f"m{rank}.pt"))
    finally:
        P.reset_tp()
        dist.destroy_process_group()


def test_tp2_llama_model_matches_unsharded():
    """The Llama adapter's full-model sharding (vocab-parallel embedding and
    head, heads split for q/k/v/o, uneven-capable MLP split) reproduces the
    unsharded logits, and with the exact input-gradient operators (including
    the one on the vocab-parallel head input) every rank's replicated-parameter
    gradients equal the unsharded ones."""
    pytest.importorskip("transformers")
    port = _free_port()
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_model_worker, args=(2, port, td), nprocs=2, join=True, start_method="spawn")
        rs = [torch.load(os.path.join(td, f"m{r}.pt")) for r in range(2)]
    m, ids, G = _tiny_llama()
    logits = m(input_ids=ids).logits
    (logits * G).sum().backward()
    for r in rs:
        v0, v1 = r["v"]
        assert torch.allclose(r["logits"], logits.detach()[..., v0:v1], rtol=1e-10, atol=1e-12)
        for n, g in r["norms"].items():
            ref = dict(m.named_parameters())[n].grad
            assert torch.allclose(g, ref, rtol=1e-9, atol=1e-12), n
        e0, e1 = r["emb_rows"]
        assert torch.allclose(r["emb_grad"], m.model.embed_tokens.weight.grad[e0:e1], rtol=1e-9, atol=1e-12)
    assert rs[0]["v"][1] == rs[1]["v"][0] and rs[1]["v"][1] == 1000


def _init_worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    from voodoo_quant import parallel as P

    r, w = P.init_tp(backend="gloo", timeout_min=2)
    res = {"rank": r, "world": w, "enabled": P.TP.enabled, "main": P.is_main_process()}
    t = torch.full((3,), float(rank + 7))
    P.tp_broadcast(t, src=1)
    res["bcast"] = t.tolist()
    gates = [torch.zeros(2, requires_grad=True), torch.zeros(3, requires_grad=True)]
    for i, g in enumerate(gates):
        g.grad = torch.arange(g.numel(), dtype=torch.float32) + 10 * i + rank
    P.all_reduce_gate_grads(gates)
    res["gates"] = [g.grad.tolist() for g in gates]
    P.barrier()
    P.tp_finalize()
    res["after"] = (P.TP.enabled, P.TP.rank, P.TP.world_size)
    torch.save(res, os.path.join(outdir, f"i{rank}.pt"))


def test_env_init_broadcast_gate_grads_and_finalize():
    """tp_init from torchrun-style env (reference parallel.py:44-96), broadcast,
    the flat gate-gradient all-reduce and tp_finalize, over gloo."""
    world = 2
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_init_worker, args=(world, _free_port(), td), nprocs=world, join=True,
                           start_method="spawn")
        rs = [torch.load(os.path.join(td, f"i{r}.pt")) for r in range(world)]
    for r, res in enumerate(rs):
        assert (res["rank"], res["world"], res["enabled"], res["main"]) == (r, world, True, r == 0)
        assert res["bcast"] == [8.0, 8.0, 8.0]
        assert res["gates"] == [[1.0, 3.0], [21.0, 23.0, 25.0]]
        assert res["after"] == (False, 0, 1)


def _qwen35(seed=0):
    from transformers.models.qwen3_5 import configuration_qwen3_5 as C, modeling_qwen3_5 as M

    cfg = C.Qwen3_5TextConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                              num_attention_heads=4, num_key_value_heads=2, head_dim=64, linear_num_key_heads=2,
                              linear_num_value_heads=4, linear_key_head_dim=64, linear_value_head_dim=64,
                              layer_types=["linear_attention", "full_attention"])
    torch.manual_seed(seed)
    return M.Qwen3_5ForCausalLM(cfg).float().eval()


def _qwen35_worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from voodoo_quant import parallel as P

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        P.adopt_process_group(0)
        m = _qwen35()
        for layer in m.model.layers:
            if hasattr(layer, "linear_attn"):
                P.tp_ssm(layer.linear_attn)
            if hasattr(layer, "self_attn"):
                P.tp_attention(layer.self_attn)
            P.tp_mlp(layer.mlp)
        x = torch.randint(0, 512, (2, 24), generator=torch.Generator().manual_seed(1))
        with torch.no_grad():
            y = m(input_ids=x, use_cache=False).logits
        gdn = m.model.layers[0].linear_attn
        torch.save({"y": y, "dims": (gdn.key_dim, gdn.value_dim, gdn.num_v_heads, gdn.conv_dim,
                                     tuple(gdn.conv1d.weight.shape))}, os.path.join(outdir, f"q{rank}.pt"))
    finally:
        P.reset_tp()
        dist.destroy_process_group()


def test_qwen35_tp2_gated_attention_and_deltanet_match_unsharded():
    """tp_attention (per-head q|gate pairs) and tp_ssm (Gated DeltaNet by
    value heads, with the depthwise conv and per-head parameters made
    rank-local) on a tiny Hugging Face Qwen3.5 text model: the TP-2 logits
    equal the unsharded model's (fp32, 1e-5 relative)."""
    pytest.importorskip("transformers.models.qwen3_5")
    world = 2
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_qwen35_worker, args=(world, _free_port(), td), nprocs=world, join=True,
                           start_method="spawn")
        rs = [torch.load(os.path.join(td, f"q{r}.pt")) for r in range(world)]
    ref_model = _qwen35()
    x = torch.randint(0, 512, (2, 24), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = ref_model(input_ids=x, use_cache=False).logits
    for r in rs:
        assert r["dims"] == (64, 128, 2, 256, (256, 1, 4))
        assert float((r["y"] - ref).norm()) <= 1e-5 * float(ref.norm())


_HEAD_LOCAL_NORMS = ("linear_attn.norm", "q_norm", "k_norm", "q_layernorm", "k_layernorm")


def _hybrid(kind: str):
    """Tiny fp64 Qwen3.5 (Gated DeltaNet + gated attention) or LFM2
    (short conv + GQA attention) causal LM with seeded weights."""
    torch.manual_seed(11)
    if kind == "qwen35":
        from transformers.models.qwen3_5 import configuration_qwen3_5 as C, modeling_qwen3_5 as M

        cfg = C.Qwen3_5TextConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                  num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                                  linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=64,
                                  linear_value_head_dim=64, layer_types=["linear_attention", "full_attention"])
        m = M.Qwen3_5ForCausalLM(cfg)
    else:
        from transformers.models.lfm2 import configuration_lfm2 as C, modeling_lfm2 as M

        cfg = C.Lfm2Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                           num_attention_heads=4, num_key_value_heads=2, layer_types=["conv", "full_attention"])
        m = M.Lfm2ForCausalLM(cfg)
    m = m.double().eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() >= 2:
                p.copy_(torch.randn_like(p) * 0.05)
    ids = torch.randint(0, 512, (2, 16), generator=torch.Generator().manual_seed(2))
    G = torch.randn(2, 16, 512, dtype=torch.float64, generator=torch.Generator().manual_seed(4))
    return m, ids, G


def _hybrid_worker(rank, world, port, outdir, kind):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from voodoo_quant import parallel as P

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        P.adopt_process_group(0)
        m, ids, G = _hybrid(kind)
        P.tp_patch_model(m, verbose=False)
        v0, v1 = m.lm_head.tp_vocab_start, m.lm_head.tp_vocab_end
        logits = m(input_ids=ids, use_cache=False).logits
        (logits * G[..., v0:v1]).sum().backward()
        norms = {n: p.grad.clone() for n, p in m.named_parameters() if "norm" in n and p.grad is not None}
        torch.save({"logits": logits.detach(), "v": (v0, v1), "norms": norms}, os.path.join(outdir, f"h{rank}.pt"))
    finally:
        P.reset_tp()
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["qwen35", "lfm2"])
def test_tp2_hybrid_adapters_match_unsharded(kind):
    """tp_patch_model through the Qwen3.5 hybrid and LFM2 adapters: the TP-2
    vocabulary-shard logits equal the unsharded model's (1e-6 relative: the
    models compute parts in fp32), and every norm applied to the full hidden
    state gets the unsharded gradient on every rank (exact input-gradient
    operators at every sharded block)."""
    pytest.importorskip(f"transformers.models.{'qwen3_5' if kind == 'qwen35' else 'lfm2'}")
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_hybrid_worker, args=(2, _free_port(), td, kind), nprocs=2, join=True,
                           start_method="spawn")
        rs = [torch.load(os.path.join(td, f"h{r}.pt")) for r in range(2)]
    m, ids, G = _hybrid(kind)
    logits = m(input_ids=ids, use_cache=False).logits
    (logits * G).sum().backward()
    ref = dict(m.named_parameters())
    for r in rs:
        v0, v1 = r["v"]
        ref_l = logits.detach()[..., v0:v1]
        assert float((r["logits"] - ref_l).norm()) <= 1e-6 * float(ref_l.norm()), \
            float((r["logits"] - ref_l).norm() / ref_l.norm())
        assert r["norms"], "no norm gradients recorded"
        for n, g in r["norms"].items():
            if not any(k in n for k in _HEAD_LOCAL_NORMS):
                assert float((g - ref[n].grad).norm()) <= 1e-5 * float(ref[n].grad.norm()) + 1e-12, n
    # per-head norms run on each rank's own heads: their gradients are
    # partial sums that add up to the unsharded one
    for n in rs[0]["norms"]:
        if any(k in n for k in _HEAD_LOCAL_NORMS):
            total = rs[0]["norms"][n] + rs[1]["norms"][n]
            assert float((total - ref[n].grad).norm()) <= 1e-5 * float(ref[n].grad.norm()) + 1e-12, n
