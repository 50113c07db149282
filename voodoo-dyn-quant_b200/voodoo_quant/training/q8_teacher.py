"""Q8_0 teacher on the B200 kernels (drop-in for training/q8_teacher.py).

The reference keeps the teacher's Q8_0 bytes on the GPU and dequantizes them
per forward with torch ops before ``F.linear`` (voodoo_quant/training/
q8_teacher.py:62-173).  Here ``Q8Linear`` is the gated path with one
candidate: ``vq_mix`` (K = 1, p = [1]) decodes the Q8_0 blocks to a bf16
weight in one HBM pass and ``vq_linear_fwd`` runs the tcgen05 GEMM; the
decoded weight is dropped after the call.  ``Q8Embedding`` decodes only the
rows the batch touches.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.nn as nn

from voodoo_quant import _C


def _q8_rows(qweight: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    return qweight.view(rows, (cols // 32) * 34)


class Q8Linear(nn.Module):
    """nn.Linear stand-in holding Q8_0 bytes; forward-only (teacher).

    ``qbytes`` holds rows of ``padded_in`` weights (default ``in_features``, a
    multiple of 256); the inputs are columns ``[in_col_offset, in_col_offset +
    in_features)`` of them -- a halo shard of a row-parallel Linear, whose
    stored blocks cover more than the rank's own columns.
    """

    def __init__(self, qbytes: torch.Tensor, out_features: int, in_features: int, bias=None, device=None,
                 padded_in: int | None = None, in_col_offset: int = 0):
        super().__init__()
        if bias is not None:
            raise NotImplementedError("Q8Linear does not support bias")
        padded = in_features if padded_in is None else padded_in
        if padded % 256:
            raise ValueError(f"Q8Linear needs in_features % 256 == 0 on this path, got {padded}")
        if in_col_offset < 0 or in_col_offset % 8 or in_col_offset + in_features > padded:
            raise ValueError(f"Q8Linear: input columns [{in_col_offset}, {in_col_offset + in_features}) "
                             f"do not fit {padded} stored columns at a multiple of 8")
        self.out_features = out_features
        self.in_features = in_features
        self.padded_in_features = padded
        self.in_col_offset = in_col_offset
        dev = torch.device(device) if device is not None else qbytes.device
        self.register_buffer("qweight", qbytes.reshape(-1, 34).to(dev).contiguous())
        self.register_buffer("_one", torch.ones(1, dtype=torch.float32, device=dev), persistent=False)

    def weight_bf16(self) -> torch.Tensor:
        off = self.in_col_offset
        w = _C.mix(["Q8_0"], [self.qweight], self._one, self.out_features, self.padded_in_features,
                   off + self.in_features)
        return w[:, off:off + self.in_features] if off else w

    @torch.no_grad()
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = self.weight_bf16()
        y = _C.linear_fwd(x.reshape(-1, self.in_features), w, self.out_features, self.in_features)
        return y.to(x.dtype).reshape(*x.shape[:-1], self.out_features)


def q8_groupable(mods) -> bool:
    """Whether teacher Linears sharing an input can run as one GEMM."""
    if len(mods) < 2:
        return False
    m0 = mods[0]
    return all(type(m) is Q8Linear and m.in_features == m0.in_features and not m.in_col_offset and
               m.out_features % 8 == 0 and m.qweight.device == m0.qweight.device for m in mods)


@torch.no_grad()
def q8_linear_group(mods, x: torch.Tensor) -> torch.Tensor:
    """x [W_1; W_2; ...]^T for teacher Linears sharing the input x (q/k/v,
    gate/up): each Q8_0 weight decoded into its row range of one bf16 weight,
    then one GEMM; layer i's outputs in its column range of the result."""
    in_f = mods[0].in_features
    ld = (in_f + 7) // 8 * 8
    n_tot = sum(m.out_features for m in mods)
    w = torch.empty(n_tot, ld, dtype=torch.bfloat16, device=mods[0].qweight.device)
    a = 0
    for m in mods:
        b = a + m.out_features
        _C.mix(["Q8_0"], [m.qweight], m._one, m.out_features, m.padded_in_features, in_f, out=w[a:b])
        a = b
    y = _C.linear_fwd(x.reshape(-1, in_f), w, n_tot, in_f)
    return y.to(x.dtype).reshape(*x.shape[:-1], n_tot)


def q8_swiglu_ok(gate, up, x: torch.Tensor) -> bool:
    """Whether a teacher MLP's gate/up pair can run as one GEMM with the
    SwiGLU in its epilogue (more than 128 tokens, a multiple of 128 features)."""
    return (q8_groupable((gate, up)) and gate.out_features == up.out_features and gate.out_features % 128 == 0
            and x.numel() // max(gate.in_features, 1) > 128)


@torch.no_grad()
def q8_swiglu_group(gate, up, x: torch.Tensor) -> torch.Tensor:
    """silu(x W_gate^T) * (x W_up^T) for a teacher MLP: both Q8_0 weights
    decoded into one bf16 [2F, Kin] weight, then one GEMM whose epilogue
    applies the SwiGLU (``vq_linear_fwd_swiglu``); the [tokens, 2F] gate|up
    output is never written.  Equal to ``q8_linear_group`` followed by the
    SwiGLU kernel."""
    in_f, F_ = gate.in_features, gate.out_features
    ld = (in_f + 7) // 8 * 8
    w = torch.empty(2 * F_, ld, dtype=torch.bfloat16, device=gate.qweight.device)
    _C.mix(["Q8_0"], [gate.qweight], gate._one, F_, gate.padded_in_features, in_f, out=w[:F_])
    _C.mix(["Q8_0"], [up.qweight], up._one, F_, up.padded_in_features, in_f, out=w[F_:])
    h = _C.linear_fwd_swiglu(x.reshape(-1, in_f), w, F_, in_f)
    return h.to(x.dtype).reshape(*x.shape[:-1], F_)


class Q8Embedding(nn.Module):
    """nn.Embedding stand-in holding Q8_0 bytes; decodes the touched rows."""

    def __init__(self, qbytes: torch.Tensor, num_embeddings: int, embedding_dim: int, device=None):
        super().__init__()
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        dev = torch.device(device) if device is not None else qbytes.device
        self.register_buffer("qweight", qbytes.reshape(-1, 34).to(dev).contiguous())
        self.register_buffer("_one", torch.ones(1, dtype=torch.float32, device=dev), persistent=False)

    @torch.no_grad()
    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        from voodoo_quant.layers import _STATIC_STATE

        if _STATIC_STATE.enabled:  # one row per token, repeats included: no host round trip
            flat = ids.reshape(-1)
            sub = _q8_rows(self.qweight, self.num_embeddings, self.embedding_dim).index_select(0, flat)
            w = _C.mix(["Q8_0"], [sub.reshape(-1)], self._one, flat.numel(), self.embedding_dim,
                       self.embedding_dim)
            return w[:, :self.embedding_dim].reshape(*ids.shape, self.embedding_dim)
        rows, inverse = torch.unique(ids.reshape(-1), return_inverse=True)
        sub = _q8_rows(self.qweight, self.num_embeddings, self.embedding_dim).index_select(0, rows)
        w = _C.mix(["Q8_0"], [sub.reshape(-1)], self._one, rows.numel(), self.embedding_dim, self.embedding_dim)
        return w[inverse].reshape(*ids.shape, self.embedding_dim)


def wrap_q8_teacher(model: nn.Module, quantizer: Callable[[torch.Tensor], torch.Tensor],
                    skip_names: Optional[set[str]] = None) -> nn.Module:
    """Replace every nn.Linear / nn.Embedding of `model` with its Q8_0 form in place.

    `quantizer(weight) -> uint8 [nblocks, 34]` produces the Q8_0 bytes (libggml
    ``quantize_tensor(w, "Q8_0")`` or the round-to-nearest packer, which is
    ggml's reference Q8_0 rule).  Mirrors ``wrap_q8_teacher``
    (q8_teacher.py:176-294) for the modules on the step's path.
    """
    skip_names = skip_names or set()
    for name, child in list(model.named_children()):
        if name in skip_names:
            continue
        if isinstance(child, nn.Linear):
            w = child.weight.data
            spec = getattr(child, "tp_shard_spec", None)
            if spec is not None and spec.halo:
                # halo shard: pack the full tensor's blocks covering the rank's columns
                full = child.tp_full_weight
                new = Q8Linear(quantizer(spec.local_block_weight(full)), child.out_features, child.in_features,
                               device=w.device, padded_in=spec.local_padded_in(full.shape[1], ["Q8_0"]),
                               in_col_offset=spec.in_col_offset)
            else:
                new = Q8Linear(quantizer(w), child.out_features, child.in_features, device=w.device)
            for attr in ("tp_shard_spec", "tp_vocab_start", "tp_vocab_end"):
                if hasattr(child, attr):
                    setattr(new, attr, getattr(child, attr))
            if hasattr(child, "tp_shard_spec") and child.tp_shard_spec.col_offset is not None:
                new = _RowParallelQ8(new)
            setattr(model, name, new)
            del child
        elif isinstance(child, nn.Embedding):
            w = child.weight.data
            new = Q8Embedding(quantizer(w), child.num_embeddings, child.embedding_dim, device=w.device)
            if hasattr(child, "tp_vocab_start"):
                new = _VocabParallelQ8(new, child.tp_vocab_start, child.num_embeddings)
            setattr(model, name, new)
            del child
        else:
            wrap_q8_teacher(child, quantizer, skip_names)
    return model


class _RowParallelQ8(nn.Module):
    def __init__(self, inner: Q8Linear):
        super().__init__()
        self.inner = inner
        self.out_features, self.in_features = inner.out_features, inner.in_features

    @torch.no_grad()
    def forward(self, x):
        from voodoo_quant.parallel import sp_enabled, tp_all_reduce_sum_
        if sp_enabled():  # partial sums: the block reduce-scatters them
            return self.inner(x)
        return tp_all_reduce_sum_(self.inner(x))


class _VocabParallelQ8(nn.Module):
    def __init__(self, inner: Q8Embedding, vocab_start: int, rows: int):
        super().__init__()
        self.inner = inner
        self.vocab_start, self.rows = vocab_start, rows

    def forward(self, ids):
        from voodoo_quant.parallel import sp_enabled, tp_all_reduce_sum_
        mask = (ids < self.vocab_start) | (ids >= self.vocab_start + self.rows)
        out = self.inner((ids - self.vocab_start).clamp(0, self.rows - 1))
        out = out * (~mask).unsqueeze(-1).to(out.dtype)
        return out if sp_enabled() else tp_all_reduce_sum_(out)
