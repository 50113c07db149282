"""Seeded synthetic workloads of the benchmark configurations.

No checkpoints or datasets are reachable offline, so the distillation step is
exercised on random-init Llama-style decoders of the configured shapes
(weights N(0, 0.02), RMSNorm weights 1), uniform random tokens, and packed
candidates from the round-to-nearest GGUF packer (``quants.rtn``), which
stands in for llama.cpp's quantiser.  The teacher is the Q8_0 round trip of
the same weights.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

ALL_K = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]


@dataclass
class ModelShape:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int
    tied: bool
    head_dim: int | None = None
    candidates: list[str] = field(default_factory=lambda: list(ALL_K))
    batch: int = 1
    seq: int = 512
    budget: float = 0.45  # compression_ratio: target bytes / 8-bit bytes
    # per-role candidate menus (the reference's --attention_candidates /
    # --non_attention_candidates, layers.py:1878-1905); None = `candidates`
    attention_candidates: list[str] | None = None
    non_attention_candidates: list[str] | None = None
    # sigma of per-row log-normal(0, sigma) scales on every weight matrix (0 = none)
    row_scale_sigma: float = 0.0


# Config 5's seven candidates in the order the configuration lists them.  Its
# menus are per role: the MLP projections, the embedding and the head choose
# among all seven (Q2_K to Q8_0), attention among the mid rungs and up
# (Q4_K, IQ4_XS, Q5_K, Q6_K, Q8_0), as the reference's own configurations
# give attention a higher menu than the MLP (configs/qwen38_27b_voodoo30_tp4.sh).
K7 = ["IQ4_XS", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "Q2_K"]
K7_ATTENTION = ["Q4_K", "IQ4_XS", "Q5_K", "Q6_K", "Q8_0"]


SHAPES = {
    # CPU-runnable tiny step
    "tiny": ModelShape(2, 256, 4, 4, 768, 4096, False, candidates=["Q4_K", "Q5_K", "Q6_K", "Q8_0"], batch=2,
                       seq=128, budget=0.45),
    # config 3: ~0.6B dense decoder, tied embeddings
    "0.6b": ModelShape(28, 1024, 16, 8, 3072, 151936, True, head_dim=128, batch=8, seq=2048, budget=0.45),
    # config 4: 8B Llama-3 shape
    "8b": ModelShape(32, 4096, 32, 8, 14336, 128256, False, batch=4, seq=4096, budget=0.30),
    # config 5: 32B dense decoder, TP-4 / TP-8 (o_proj at TP-8 is a halo shard:
    # 5 heads x 128 = 640 columns per rank; down_proj splits 13/12 blocks)
    "32b": ModelShape(64, 5120, 40, 8, 25600, 152064, False, head_dim=128, candidates=list(K7), batch=2,
                      seq=8192, budget=0.30, attention_candidates=list(K7_ATTENTION),
                      non_attention_candidates=list(K7), row_scale_sigma=0.5),
}


def llama_config(shape: ModelShape):
    from transformers import LlamaConfig

    kw = dict(vocab_size=shape.vocab, hidden_size=shape.hidden, intermediate_size=shape.ffn,
              num_hidden_layers=shape.layers, num_attention_heads=shape.heads,
              num_key_value_heads=shape.kv_heads, rms_norm_eps=1e-6, rope_theta=1e4,
              tie_word_embeddings=shape.tied, max_position_embeddings=max(shape.seq, 256),
              attention_bias=False, mlp_bias=False)
    if shape.head_dim is not None:
        kw["head_dim"] = shape.head_dim
    cfg = LlamaConfig(**kw)
    cfg._attn_implementation = "sdpa"
    return cfg


def build_llama(shape: ModelShape, device, dtype=torch.bfloat16, seed: int = 0):
    """Random-init LlamaForCausalLM on `device`: every weight N(0, 0.02), norms 1.
    With ``shape.row_scale_sigma`` > 0, each row of every weight matrix is then
    scaled by its own log-normal(0, sigma) factor (drawn right after the
    matrix, from the same generator)."""
    from transformers import LlamaForCausalLM
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    cfg = llama_config(shape)
    with torch.device("meta"):
        model = LlamaForCausalLM(cfg)
    model = model.to_empty(device=device).to(dtype)
    g = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm.weight"):
                p.fill_(1.0)
            else:
                p.copy_(torch.randn(p.shape, generator=g, device=device, dtype=torch.float32).to(dtype) * 0.02)
                if shape.row_scale_sigma > 0 and p.dim() == 2:
                    z = torch.randn(p.shape[0], 1, generator=g, device=device, dtype=torch.float32)
                    p.copy_((p.float() * torch.exp(z * shape.row_scale_sigma)).to(dtype))
    model.model.rotary_emb = LlamaRotaryEmbedding(cfg, device=device)
    if shape.tied:
        model.tie_weights()
    return model


def rtn_candidate_provider(name: str, weight: torch.Tensor, types: list[str]) -> dict:
    """Packed candidates of a (256-padded) weight via the round-to-nearest packer."""
    from voodoo_quant.quants import rtn

    w = weight.detach().to(torch.float32)
    return {qt: rtn.quantize(w, qt) for qt in types}


def q8_quantizer(weight: torch.Tensor) -> torch.Tensor:
    """Q8_0 teacher bytes: the sm_100a quantiser on CUDA weights, the same
    rule in torch elsewhere (both ggml's reference Q8_0 rule)."""
    if weight.is_cuda:
        from voodoo_quant import _C

        return _C.quantize(weight.detach(), "Q8_0")
    from voodoo_quant.quants import rtn

    return rtn.quantize(weight.detach().to(torch.float32), "Q8_0")


def random_tokens(shape: ModelShape, device, seed: int = 1, batch: int | None = None, seq: int | None = None):
    g = torch.Generator(device=device).manual_seed(seed)
    b = batch or shape.batch
    s = seq or shape.seq
    x = torch.randint(0, shape.vocab, (b, s), device=device, generator=g)
    y = torch.randint(0, shape.vocab, (b, s), device=device, generator=g)
    return x, y
