"""Fused elementwise work of the Llama decoder block for the distillation step.

The reference's step runs the Hugging Face Llama block around the gated
Linears (voodoo_quant/training/trainer.py:2538-2556).  In that block the
RMSNorm (fp32 cast, pow, mean, rsqrt, two multiplies), the rotary embedding
(rotate_half's neg + cat, two multiplies and an add on the transposed q/k
views) and the SwiGLU product run as separate torch kernels, forward and
backward: a third of an 8B step's device time and over half of a 0.6B step's.
``fuse_llama_blocks`` routes those three through one-pass CUDA kernels of
``libvoodoo_b200`` (``vq_rmsnorm_fwd/bwd``, ``vq_rope``,
``vq_swiglu_fwd/bwd``).  The attention itself stays torch's
``scaled_dot_product_attention`` (cuDNN on B200), called as the Hugging Face
``sdpa`` path calls it for a causal, unpadded, cache-free training batch.

A patched module uses the fused kernels only for CUDA bf16 activations in
that training case; any other call (a KV cache, an explicit attention mask,
other dtypes or devices) runs the module's original forward unchanged.
"""

from __future__ import annotations

import types

import torch
import torch.nn.functional as F
from torch.autograd import Function

from voodoo_quant import _C


class _RMSNormFn(Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, weight: torch.Tensor, eps: float):
        D = x.shape[-1]
        x2 = x.reshape(-1, D)
        y, rstd = _C.rmsnorm_fwd(x2, weight, eps)
        ctx.save_for_backward(x2, weight, rstd)
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, gy: torch.Tensor):
        x2, weight, rstd = ctx.saved_tensors
        g2 = gy.reshape(-1, x2.shape[1])
        dx = _C.rmsnorm_bwd(x2, g2, weight, rstd) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            n = (x2.float() * rstd[:, None]).to(torch.bfloat16).float()
            dw = (g2.float() * n).sum(0).to(weight.dtype)
        return (dx.view(gy.shape) if dx is not None else None), dw, None


class _AddRMSNormFn(Function):
    """h = a + res and y = RMSNorm(h) in one kernel (a decoder layer's
    residual add and the norm after it).  Backward: both inputs get the
    norm's input gradient plus the gradient reaching h directly, summed in
    fp32 inside the norm's backward kernel."""

    @staticmethod
    def forward(ctx, a: torch.Tensor, res: torch.Tensor, weight: torch.Tensor, eps: float):
        D = a.shape[-1]
        h, y, rstd = _C.add_rmsnorm_fwd(a.reshape(-1, D), res.reshape(-1, D), weight, eps)
        ctx.save_for_backward(h, weight, rstd)
        return h.view(a.shape), y.view(a.shape)

    @staticmethod
    def backward(ctx, gh: torch.Tensor, gy: torch.Tensor):
        h, weight, rstd = ctx.saved_tensors
        D = h.shape[1]
        gy2 = gy.reshape(-1, D)
        dx = None
        if ctx.needs_input_grad[0] or ctx.needs_input_grad[1]:
            dx = _C.rmsnorm_bwd_add(h, gy2, gh.reshape(-1, D), weight, rstd).view(gy.shape)
        dw = None
        if ctx.needs_input_grad[2]:
            n = (h.float() * rstd[:, None]).to(torch.bfloat16).float()
            dw = (gy2.float() * n).sum(0).to(weight.dtype)
        return (dx if ctx.needs_input_grad[0] else None), (dx if ctx.needs_input_grad[1] else None), dw, None


class _RopeFn(Function):
    """q [B, S, Hq, D], k [B, S, Hk, D] -> rotated, contiguous [B, S, H, D]."""

    @staticmethod
    def forward(ctx, q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        qo, ko = _C.rope(q, k, cos, sin)
        ctx.save_for_backward(cos, sin)
        return qo, ko

    @staticmethod
    def backward(ctx, gq: torch.Tensor, gk: torch.Tensor):
        cos, sin = ctx.saved_tensors
        dq, dk = _C.rope(gq, gk, cos, sin, backward=True)
        return dq, dk, None, None


class _SwiGLUFn(Function):
    @staticmethod
    def forward(ctx, gate: torch.Tensor, up: torch.Tensor):
        F_ = gate.shape[-1]
        g2, u2 = gate.reshape(-1, F_), up.reshape(-1, F_)
        y = _C.swiglu_fwd(g2, u2)
        ctx.save_for_backward(g2, u2)
        ctx.shape = gate.shape
        return y.view(gate.shape)

    @staticmethod
    def backward(ctx, gy: torch.Tensor):
        g2, u2 = ctx.saved_tensors
        dg, du = _C.swiglu_bwd(g2, u2, gy.reshape(-1, g2.shape[1]))
        return dg.view(ctx.shape), du.view(ctx.shape)


class _SwiGLUPairFn(Function):
    """silu(gate) * up of a grouped gate|up projection output [..., 2F]; the
    backward writes d gate and d up into one [rows, 2F] gradient, the layout
    the grouped projection's backward reads."""

    @staticmethod
    def forward(ctx, gu: torch.Tensor):
        F_ = gu.shape[-1] // 2
        g2 = gu.reshape(-1, 2 * F_)
        y = _C.swiglu_fwd(g2[:, :F_], g2[:, F_:])
        ctx.save_for_backward(g2)
        ctx.shape = gu.shape
        return y.view(*gu.shape[:-1], F_)

    @staticmethod
    def backward(ctx, gy: torch.Tensor):
        (g2,) = ctx.saved_tensors
        F_ = g2.shape[1] // 2
        dgu = torch.empty(g2.shape, dtype=torch.bfloat16, device=g2.device)
        _C.swiglu_bwd(g2[:, :F_], g2[:, F_:], gy.reshape(-1, F_), out=dgu)
        return dgu.view(ctx.shape)


def _group_projection(mods, x: torch.Tensor):
    """Linears that read the same input as one GEMM when they allow it (gated
    student layers or Q8_0 teacher layers); None otherwise."""
    from voodoo_quant.layers import gated_linear_group, groupable
    from voodoo_quant.training.q8_teacher import q8_groupable, q8_linear_group

    if groupable(mods):
        return gated_linear_group(mods, x)
    if q8_groupable(mods):
        return q8_linear_group(mods, x)
    return None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return _RMSNormFn.apply(x, weight, eps)


def add_rms_norm(a: torch.Tensor, res: torch.Tensor, weight: torch.Tensor, eps: float):
    """(a + res, RMSNorm(a + res)) for bf16 [..., D] tensors."""
    return _AddRMSNormFn.apply(a, res, weight, eps)


def rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    return _RopeFn.apply(q, k, cos, sin)


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return _SwiGLUFn.apply(gate, up)


def _fusable(x: torch.Tensor) -> bool:
    return x.is_cuda and x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0


def _rmsnorm_forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
    if not (_fusable(hidden_states) and self.weight.dtype == torch.bfloat16 and hidden_states.shape[-1] <= 8192):
        return self._vq_orig_forward(hidden_states)
    return rms_norm(hidden_states, self.weight, self.variance_epsilon)


def _mlp_forward(self, x: torch.Tensor) -> torch.Tensor:
    if not _fusable(x):
        return self._vq_orig_forward(x)
    if not torch.is_grad_enabled():  # a forward-only (teacher) MLP: SwiGLU in the gate|up GEMM's epilogue
        from voodoo_quant.training.q8_teacher import q8_swiglu_group, q8_swiglu_ok

        if q8_swiglu_ok(self.gate_proj, self.up_proj, x):
            return self.down_proj(q8_swiglu_group(self.gate_proj, self.up_proj, x))
    if self.gate_proj.out_features == self.up_proj.out_features:
        gu = _group_projection((self.gate_proj, self.up_proj), x)
        if gu is not None and _fusable(gu):
            return self.down_proj(_SwiGLUPairFn.apply(gu))
    g = self.gate_proj(x)
    u = self.up_proj(x)
    if not (_fusable(g) and g.shape == u.shape):
        return self.down_proj(self.act_fn(g) * u)
    return self.down_proj(swiglu(g, u))


def _attention_forward(self, hidden_states: torch.Tensor, position_embeddings=None, attention_mask=None,
                       past_key_values=None, **kwargs):
    if getattr(self, "_vq_causal_batches", False) and past_key_values is None:
        # batches of the distillation step are causal and unpadded: the only
        # mask Hugging Face builds for them is the causal one, which it
        # materialises while a CUDA graph records instead of leaving it to
        # is_causal
        attention_mask = None
    if (past_key_values is not None or attention_mask is not None or position_embeddings is None
            or not _fusable(hidden_states) or self.head_dim % 16 or kwargs.get("output_attentions", False)):
        return self._vq_orig_forward(hidden_states, position_embeddings=position_embeddings,
                                     attention_mask=attention_mask, past_key_values=past_key_values, **kwargs)
    B, S = hidden_states.shape[:2]
    qkv = _group_projection((self.q_proj, self.k_proj, self.v_proj), hidden_states)
    if qkv is not None:  # one GEMM; q, k, v are column ranges of its output
        nq, nk = self.q_proj.out_features, self.k_proj.out_features
        # split, not three slices: its backward concatenates the three
        # gradients in one pass (a slice's backward zero-fills a full-size
        # gradient per slice and autograd adds the three)
        q, k, v = qkv.split([nq, nk, qkv.shape[-1] - nq - nk], dim=-1)
        q = q.view(B, S, -1, self.head_dim)
        k = k.view(B, S, -1, self.head_dim)
        v = v.view(B, S, -1, self.head_dim)
    else:
        q = self.q_proj(hidden_states).view(B, S, -1, self.head_dim)
        k = self.k_proj(hidden_states).view(B, S, -1, self.head_dim)
        v = self.v_proj(hidden_states).view(B, S, -1, self.head_dim)
    cos, sin = position_embeddings
    q, k = rope(q, k, cos, sin)
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=S > 1,
                                       scale=self.scaling, enable_gqa=q.shape[2] != k.shape[2])
    o = o.transpose(1, 2).reshape(B, S, -1)
    return self.o_proj(o), None


def _sp_decoder(self, h: torch.Tensor, position_embeddings, shape) -> torch.Tensor:
    """One decoder layer under sequence parallelism: ``h`` is this rank's
    [tokens / N, hidden] shard of the residual stream (tokens of the
    flattened [B, S] batch, ranks in order).  The RMSNorms and residual adds
    run on the shard; each block all-gathers its normalised input, runs its
    column-parallel projections, attention (whole sequences, this rank's
    heads) or SwiGLU, and its row-parallel projection on all tokens, and
    reduce-scatters the partial output back to the shard."""
    from voodoo_quant.parallel import sp_gather, sp_scatter

    B, S = shape
    norm = self.post_attention_layernorm
    x = self.input_layernorm(h)
    a, _ = self.self_attn(hidden_states=sp_gather(x).view(B, S, -1), position_embeddings=position_embeddings,
                          attention_mask=None)
    a = sp_scatter(a.reshape(B * S, -1))
    if _fusable(a) and getattr(norm, "weight", None) is not None and norm.weight.dtype == torch.bfloat16 \
            and hasattr(norm, "variance_epsilon") and a.shape[-1] <= 8192:
        h, x = add_rms_norm(a, h, norm.weight, norm.variance_epsilon)
    else:
        h = h + a
        x = norm(h)
    m = self.mlp(sp_gather(x).view(B, S, -1))
    return h + sp_scatter(m.reshape(B * S, -1))


def _decoder_forward(self, hidden_states: torch.Tensor, attention_mask=None, position_ids=None,
                     past_key_values=None, use_cache=False, position_embeddings=None, sp_shape=None, **kwargs):
    """Hugging Face LlamaDecoderLayer.forward with the residual add after the
    attention fused into the post-attention RMSNorm (``sp_shape`` = (B, S):
    the sequence-parallel layer, ``_sp_decoder``)."""
    if sp_shape is not None:
        return _sp_decoder(self, hidden_states, position_embeddings, sp_shape)
    norm = self.post_attention_layernorm
    if not (_fusable(hidden_states) and getattr(norm, "weight", None) is not None
            and norm.weight.dtype == torch.bfloat16 and hasattr(norm, "variance_epsilon")
            and hidden_states.shape[-1] <= 8192):
        return self._vq_orig_forward(hidden_states, attention_mask=attention_mask, position_ids=position_ids,
                                     past_key_values=past_key_values, use_cache=use_cache,
                                     position_embeddings=position_embeddings, **kwargs)
    residual = hidden_states
    x = self.input_layernorm(hidden_states)
    x, _ = self.self_attn(hidden_states=x, attention_mask=attention_mask, position_ids=position_ids,
                          past_key_values=past_key_values, use_cache=use_cache,
                          position_embeddings=position_embeddings, **kwargs)
    if _fusable(x) and x.shape == residual.shape:
        h, x = add_rms_norm(x, residual, norm.weight, norm.variance_epsilon)
    else:
        h = residual + x
        x = norm(h)
    return h + self.mlp(x)


def _norm_weights_fusable(norm) -> bool:
    w = getattr(norm, "weight", None)
    return (w is not None and w.is_cuda and w.dtype == torch.bfloat16 and hasattr(norm, "variance_epsilon")
            and w.shape[-1] % 8 == 0 and w.shape[-1] <= 8192)


def _chained_model_forward(self, input_ids=None, attention_mask=None, position_ids=None, past_key_values=None,
                           inputs_embeds=None, use_cache=None, **kwargs):
    """Hugging Face LlamaModel.forward for whole causal batches (the
    distillation step) with every residual add fused into the RMSNorm that
    reads its sum: a layer hands its MLP output on unsummed, and the next
    layer's input norm (or the final norm) adds it to the residual stream
    and normalises in one kernel, as the post-attention norm already does.
    Values are those of the layer-by-layer forward (the same bf16 sums, the
    same norms); anything else goes to the stock forward."""
    from transformers.modeling_outputs import BaseModelOutputWithPast

    from voodoo_quant.parallel import sp_enabled

    plain = (sp_enabled() or input_ids is None or inputs_embeds is not None or past_key_values is not None
             or use_cache or attention_mask is not None or position_ids is not None
             or kwargs.get("cache_position") is not None
             or any(kwargs.get(k) for k in ("output_hidden_states", "output_attentions")))
    layers = self.layers[: self.config.num_hidden_layers]
    if not plain:
        plain = not (_norm_weights_fusable(self.norm) and all(
            hasattr(l, "_vq_orig_forward") and hasattr(l.self_attn, "_vq_orig_forward")
            and hasattr(l.mlp, "_vq_orig_forward") and _norm_weights_fusable(l.input_layernorm)
            and _norm_weights_fusable(l.post_attention_layernorm) for l in layers))
    if plain:
        return self._vq_chain_orig_forward(input_ids=input_ids, attention_mask=attention_mask,
                                           position_ids=position_ids, past_key_values=past_key_values,
                                           inputs_embeds=inputs_embeds, use_cache=use_cache, **kwargs)
    h = self.embed_tokens(input_ids)
    S = h.shape[1]
    pe = self.rotary_emb(h, position_ids=torch.arange(S, device=h.device).unsqueeze(0))
    if not _fusable(h):  # not the bf16 stream the norms expect: layer by layer
        for layer in layers:
            h = layer(h, position_embeddings=pe)
        return BaseModelOutputWithPast(last_hidden_state=self.norm(h))
    pending = None  # the previous layer's MLP output, not yet added to h
    for layer in layers:
        n1, n2 = layer.input_layernorm, layer.post_attention_layernorm
        if pending is None:
            x = rms_norm(h, n1.weight, n1.variance_epsilon)
        else:
            h, x = add_rms_norm(pending, h, n1.weight, n1.variance_epsilon)
        a, _ = layer.self_attn(hidden_states=x, attention_mask=None, position_embeddings=pe)
        h, x = add_rms_norm(a, h, n2.weight, n2.variance_epsilon)
        pending = layer.mlp(x)
    if pending is None:
        out = rms_norm(h, self.norm.weight, self.norm.variance_epsilon)
    else:
        _, out = add_rms_norm(pending, h, self.norm.weight, self.norm.variance_epsilon)
    return BaseModelOutputWithPast(last_hidden_state=out)


def fuse_llama_blocks(model: torch.nn.Module, causal_batches: bool = False) -> int:
    """Route the RMSNorm, attention (rotary) and MLP (SwiGLU) modules of a
    Hugging Face Llama model through the fused kernels, and each decoder
    layer's post-attention residual add into its RMSNorm, in place; returns
    the number of modules patched.  Idempotent.  ``causal_batches``: the
    caller only ever feeds whole causal sequences without padding (the
    distillation step), so the attention ignores the causal mask Hugging Face
    passes while a CUDA graph records and keeps the fused path, and the
    LlamaModel forward chains every residual add into the next RMSNorm
    (``_chained_model_forward``)."""
    from transformers.models.llama import modeling_llama as L

    table = ((L.LlamaRMSNorm, _rmsnorm_forward), (L.LlamaAttention, _attention_forward),
             (L.LlamaMLP, _mlp_forward), (L.LlamaDecoderLayer, _decoder_forward))
    n = 0
    for m in model.modules():
        for cls, fwd in table:
            if type(m) is cls and not hasattr(m, "_vq_orig_forward"):
                if cls is L.LlamaMLP and getattr(m.config, "hidden_act", "silu") not in ("silu", "swish"):
                    continue
                m._vq_orig_forward = m.forward
                m.forward = types.MethodType(fwd, m)
                n += 1
        if type(m) is L.LlamaAttention and causal_batches:
            m._vq_causal_batches = True
        if type(m) is L.LlamaModel and causal_batches and not hasattr(m, "_vq_chain_orig_forward"):
            m._vq_chain_orig_forward = m.forward
            m.forward = types.MethodType(_chained_model_forward, m)
            n += 1
    return n


def _sp_model_forward(self, input_ids=None, attention_mask=None, position_ids=None, past_key_values=None,
                      inputs_embeds=None, use_cache=None, **kwargs):
    """Hugging Face LlamaModel.forward for the distillation step under
    sequence parallelism: the vocabulary-parallel embedding's partial sums are
    reduce-scattered into token shards, the decoder layers run on the shards
    (``_sp_decoder``), the final RMSNorm on the shard, and the normalised
    hidden states of all tokens are all-gathered for the vocabulary-parallel
    head.  Causal, unpadded, cache-free batches only."""
    from transformers.modeling_outputs import BaseModelOutputWithPast

    from voodoo_quant.parallel import sp_enabled, sp_gather, sp_scatter

    if not sp_enabled():
        return self._vq_sp_orig_forward(input_ids=input_ids, attention_mask=attention_mask,
                                        position_ids=position_ids, past_key_values=past_key_values,
                                        inputs_embeds=inputs_embeds, use_cache=use_cache, **kwargs)
    if input_ids is None or inputs_embeds is not None or past_key_values is not None or use_cache or \
            attention_mask is not None:
        raise ValueError("sequence parallelism runs whole causal batches from input_ids only "
                         "(no attention mask, cache or inputs_embeds)")
    e = self.embed_tokens(input_ids)
    B, S, H = e.shape
    h = sp_scatter(e.reshape(B * S, H))
    pos = torch.arange(S, device=e.device).unsqueeze(0) if position_ids is None else position_ids
    pe = self.rotary_emb(e, position_ids=pos)
    for layer in self.layers[: self.config.num_hidden_layers]:
        h = layer(h, position_embeddings=pe, sp_shape=(B, S))
    h = self.norm(h)
    return BaseModelOutputWithPast(last_hidden_state=sp_gather(h).view(B, S, H))


def use_sequence_parallel(model: torch.nn.Module) -> int:
    """Let a tensor-parallel Hugging Face Llama model run sequence parallel
    while ``parallel.enable_sequence_parallel`` is on: its LlamaModel forward
    becomes ``_sp_model_forward`` and every decoder layer's forward
    ``_decoder_forward`` (the layers of ``fuse_llama_blocks``, also where the
    fused kernels do not apply).  Idempotent; returns the number of modules
    patched."""
    from transformers.models.llama import modeling_llama as L

    n = 0
    for m in model.modules():
        if type(m) is L.LlamaModel and not hasattr(m, "_vq_sp_orig_forward"):
            m._vq_sp_orig_forward = m.forward
            m.forward = types.MethodType(_sp_model_forward, m)
            n += 1
        elif type(m) is L.LlamaDecoderLayer and not hasattr(m, "_vq_orig_forward"):
            m._vq_orig_forward = m.forward
            m.forward = types.MethodType(_decoder_forward, m)
            n += 1
    return n
