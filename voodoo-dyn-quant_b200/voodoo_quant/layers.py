"""Gated mixed-quant layers on the B200 kernels (drop-in for voodoo_quant/layers.py).

``MixedQuantLinear`` / ``MixedQuantEmbedding`` keep the reference's
constructor, methods and attributes (voodoo_quant/layers.py:1640-1842): K
learnable gates, p = softmax(gates / tau), an effective weight
W_mix = sum_k p_k W_k over K packed GGUF candidates, and argmax hard
assignment after training.  What changes is where the work happens:

* The K candidates stay packed (GGUF blocks) in one HBM arena per tensor
  (``voodoo_quant.cache.pack_arena``); nothing dequantised is stored.
* Forward: ``vq_mix`` decodes the K candidates bit-exactly and writes W_mix
  once (bf16), ``vq_linear_fwd`` runs the tcgen05 GEMM.
* Backward: ``vq_linear_dx`` reuses W_mix for dX; ``vq_gategrad`` computes
  g_k = <dY^T X, W_k> in the dW GEMM's epilogue without materialising dW.
  Autograd then applies the softmax Jacobian to reach the gates, exactly as
  in the reference (``_MixedWeightFunction.backward``, :355-363).

The candidate cache on disk keeps the reference format and paths
(``_combined_cache_path``, ``_tensor_hash``, :884-943): a ``combined_lazy``
file holding {qtype: uint8 [nblocks, block_bytes]} per tensor.  Missing
candidates are quantised by libggml as in the reference (:1282-1340).
"""

from __future__ import annotations

import hashlib
import os
from pathlib import Path
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd import Function

import voodoo_quant
from voodoo_quant import _C
from voodoo_quant.cache import STORE, arena_views, pack_arena
from voodoo_quant.ggml import GPU_FORMATS, bytes_per_weight, get_quant_info, quantize_tensor

CANDIDATE_CACHE_DIR = Path(voodoo_quant.__file__).resolve().parent.parent / ".cache" / "mixed_quant_candidates"
_CANDIDATE_CACHE_ROOT = CANDIDATE_CACHE_DIR

# Keep W_mix from the forward for the backward's dX (one bf16 [out, in] per
# layer).  False recomputes it in the backward (one more HBM-bound mix pass).
KEEP_MIXED_WEIGHT = True

# SMs the gate-gradient GEMM leaves free while the layer's input-gradient
# all-reduce (reduce_input_grad under TP) is in flight, so that the two run
# concurrently; match it to the collective's CTA count (NCCL channels).
GATEGRAD_SM_RESERVE = 0

# Row chunks of dX in a layer that all-reduces its own input gradient
# (reduce_input_grad under TP): the all-reduce of chunk i runs while chunk
# i + 1 and the gate-gradient GEMM are computed.  1 = one dX GEMM.
INPUT_GRAD_CHUNKS = 1


# --------------------------------------------------------------------------- per-token quant routing
class _PTQRState:
    """Per-Token Quant Routing (reference voodoo_quant/layers.py:848-865).

    When enabled, every gated layer runs each token through ONE candidate,
    sampled from the gate probabilities, instead of the candidate mixture;
    the backward stays the mixture's straight-through Jacobian.
    """

    enabled: bool = False


_PTQR_STATE = _PTQRState()


def set_ptqr(enabled: bool) -> None:
    _PTQR_STATE.enabled = bool(enabled)


# --------------------------------------------------------------------------- static shapes
class _StaticState:
    """Static-shape mode (off by default): no host round trip and no
    data-dependent shape in the step's host code, so that the whole forward
    and backward can be recorded as one CUDA graph.  Embedding lookups then
    decode one row per token, repeats included, instead of the unique rows
    (``torch.unique`` reads its output size on the host); a vocabulary shard
    looks every token up at a clamped row and zeroes the rows that belong to
    other shards instead of gathering its own tokens (boolean indexing).
    Values are unchanged: the gated embedding's backward is a dot product per
    candidate, whose terms are the same per token either way.  Under PTQR the
    embedding draws one candidate for every row of its table (the reference
    draws one per unique row it touches, layers.py:1810-1813: the same
    distribution) and selects each token's row among the K decodes with a
    mask instead of gathering the rows of each candidate."""

    enabled: bool = False


_STATIC_STATE = _StaticState()


def set_static_shapes(enabled: bool) -> None:
    _STATIC_STATE.enabled = bool(enabled)


# --------------------------------------------------------------------------- ST-Gumbel switches
# The reference's straight-through Gumbel hardening (layers.py:821-846,
# trainer --st_gumbel) routes a fraction of tokens through hard one-hot
# candidates.  No benchmark configuration uses it and this path does not
# implement it; the switches keep the reference's names so its trainer
# imports and runs unchanged with the feature off, and turning it on fails
# loudly instead of silently training something else.
class _STGumbelState:
    enabled = False
    fraction = 0.0
    gs_tau = 1.0
    f_start = None
    f_end = None
    total_steps = 1
    step = 0


_ST_GUMBEL_STATE = _STGumbelState()


def set_st_gumbel(enabled: bool, fraction: float = 0.0, gs_tau: float = 1.0) -> None:
    if enabled:
        raise NotImplementedError("ST-Gumbel hardening is not implemented on the B200 path; use PTQR (set_ptqr)")
    _ST_GUMBEL_STATE.enabled = False
    _ST_GUMBEL_STATE.fraction = float(fraction)
    _ST_GUMBEL_STATE.gs_tau = float(gs_tau)


def set_st_gumbel_anneal(f_start: float, f_end: float, total_steps: int) -> None:
    _ST_GUMBEL_STATE.f_start = float(f_start)
    _ST_GUMBEL_STATE.f_end = float(f_end)
    _ST_GUMBEL_STATE.total_steps = max(int(total_steps), 1)


def st_gumbel_step(step: int) -> None:
    _ST_GUMBEL_STATE.step = int(step)


# --------------------------------------------------------------------------- diagnostics and helpers
def _heap_census(signum, frame) -> None:
    """SIGUSR1: print live Python objects by type and CPU tensor bytes by dtype
    (the reference's host-memory census, layers.py:225-274)."""
    import collections
    import gc

    by_type, cpu_bytes = collections.Counter(), collections.Counter()
    for obj in gc.get_objects():
        try:
            by_type[type(obj).__name__] += 1
            if torch.is_tensor(obj) and obj.device.type == "cpu":
                cpu_bytes[str(obj.dtype)] += obj.numel() * obj.element_size()
        except Exception:
            pass
    lines = ["[heap-dump] top types:"] + [f"  {n}: {c}" for n, c in by_type.most_common(12)]
    lines += ["[heap-dump] cpu tensor bytes by dtype:"] + [f"  {n}: {c}" for n, c in cpu_bytes.most_common(8)]
    print("\n".join(lines), flush=True)


def install_heap_dump_handler() -> None:
    """Arm the SIGUSR1 heap census (a no-op where signals cannot be set)."""
    try:
        import signal

        signal.signal(signal.SIGUSR1, _heap_census)
    except Exception:
        pass


def _format_duration(seconds: float | None) -> str:
    """Short duration text ('4.2s', '2m03s', '1h07m'); '...' when unknown."""
    if seconds is None or seconds != seconds or seconds == float("inf"):
        return "..."
    seconds = max(float(seconds), 0.0)
    if seconds < 60:
        return f"{seconds:.1f}s"
    m, s_ = divmod(int(seconds), 60)
    if m < 60:
        return f"{m}m{s_:02d}s"
    h, m = divmod(m, 60)
    return f"{h}h{m:02d}m"


def _quant_info_for(quant_type: str):
    """Block size / bytes of a quant type (reference layers.py:293-295)."""
    return get_quant_info(quant_type)


def dequantize_tensor_gpu(qweight: torch.Tensor, quant_type: str, out_features: int, in_features: int,
                          device) -> torch.Tensor:
    """Packed blocks -> bf16 [out_features, in_features] on `device`
    (reference layers.py:298-319): the sm_100a decoder for the B200 formats,
    the host decoder (libggml) for the others, as the reference falls back."""
    device = torch.device(device)
    if quant_type in GPU_FORMATS and device.type == "cuda":
        w = _C.dequant(qweight.to(device), quant_type, out_features, in_features)
    else:
        from voodoo_quant.ggml import dequantize_tensor

        w = dequantize_tensor(qweight.cpu(), quant_type, out_features, in_features).to(device)
    return w[:, :in_features].to(torch.bfloat16)


def _sample_token_routing(probs: torch.Tensor, num_tokens: int) -> torch.Tensor:
    """k*(t) ~ Categorical(probs) per token by Gumbel-argmax (reference :868-881).

    The same torch operations as the reference, so a given generator state
    yields the same routing.
    """
    u = torch.rand(probs.shape[0], num_tokens, device=probs.device)
    gumbel = -torch.log((-torch.log(u.clamp_min(1e-9))).clamp_min(1e-9))
    scores = torch.log(probs.clamp_min(1e-9)).unsqueeze(1) + gumbel
    return scores.argmax(dim=0)


# --------------------------------------------------------------------------- cache helpers
def _tensor_hash(t: torch.Tensor | None) -> str:
    """SHA-256 (first 16 hex) of the tensor's float32 bytes, streamed in 4M-element chunks.

    Same key as the reference (voodoo_quant/layers.py:884-908) so an existing
    candidate cache is found.
    """
    if t is None:
        return "none"
    flat = t.detach().contiguous().cpu().reshape(-1)
    h = hashlib.sha256()
    ch = 1 << 22
    for i in range(0, flat.numel(), ch):
        h.update(flat[i:i + ch].to(torch.float32).numpy().tobytes())
    return h.hexdigest()[:16]


def _safe_name(tensor_name: str) -> str:
    return tensor_name.replace(".", "_").replace("/", "_")


def _candidate_cache_path(tensor_name: str, candidate_type: str, mode: str, weight_hash: str,
                          imatrix_hash: str) -> Path:
    d = _CANDIDATE_CACHE_ROOT / _safe_name(tensor_name)
    d.mkdir(parents=True, exist_ok=True)
    return d / f"{candidate_type}_{mode}_w{weight_hash}_i{imatrix_hash}.pt"


def _combined_cache_path(tensor_name: str, mode: str, weight_hash: str, imatrix_hash: str) -> Path:
    d = _CANDIDATE_CACHE_ROOT / _safe_name(tensor_name)
    d.mkdir(parents=True, exist_ok=True)
    return d / f"combined_{mode}_w{weight_hash}_i{imatrix_hash}.pt"


def _load_cache_file(path: Path, tensor_name: str):
    """A candidate-cache file, memory-mapped; an unreadable one (truncated,
    not a torch file) is an error that names it rather than a silent
    re-quantisation or torch's bare message."""
    try:
        return torch.load(path, weights_only=True, map_location="cpu", mmap=True)
    except Exception as e:
        raise RuntimeError(f"{tensor_name}: candidate cache file {path} cannot be read ({e}); "
                           "delete it to quantize the candidates again") from e


def _atomic_torch_save(obj, path: Path) -> None:
    tmp = path.with_suffix(path.suffix + f".tmp{os.getpid()}")
    torch.save(obj, tmp)
    os.replace(tmp, path)


def _pad_weight_and_imatrix(weight: torch.Tensor, imatrix: torch.Tensor | None):
    """Zero-pad in_features to a multiple of 256 (imatrix padded with 1.0)."""
    orig_in = weight.shape[1]
    if orig_in % 256 == 0:
        return weight, imatrix, orig_in
    pad = 256 - orig_in % 256
    padded = F.pad(weight, (0, pad), "constant", 0)
    pim = None
    if imatrix is not None:
        pim = F.pad(imatrix.to(torch.float32).contiguous(), (0, pad), "constant", 1.0)
    return padded, pim, orig_in


pad_weight_and_imatrix = _pad_weight_and_imatrix


def _padded(n: int) -> int:
    return (n + 255) // 256 * 256


# --------------------------------------------------------------------------- autograd functions
class _GatedLinearFunction(Function):
    """y = x W_mix^T with W_mix = sum_k p_k W_k; gradients for x and p."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, probs: torch.Tensor, layer: "MixedQuantLinear", reducer=None):
        in_f, out_f = layer.in_features, layer.out_features
        x2 = _C._as_operand(x.reshape(-1, in_f))
        w_mix = layer._mix(probs)
        if reducer is not None:  # row-parallel: the output sum over the TP ranks, reduced in the GEMM
            y = reducer.linear(x2, w_mix, out_f, in_f)
        else:
            y = _C.linear_fwd(x2, w_mix, out_f, in_f)
        ctx.layer = layer
        ctx.x_shape = x.shape
        ctx.x_dtype = x.dtype
        ctx.save_for_backward(x2, probs)
        ctx.w_mix = w_mix if KEEP_MIXED_WEIGHT else None
        return y.to(x.dtype).reshape(*x.shape[:-1], out_f)

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        dx, dprobs = _gated_linear_backward(ctx, dy)
        return dx, dprobs, None, None


def _overlap_sms() -> int:
    """SMs a GEMM leaves free while a TP collective runs beside it."""
    from voodoo_quant.parallel import TP
    if not TP.enabled:
        return 0
    return GATEGRAD_SM_RESERVE if GATEGRAD_SM_RESERVE > 0 else TP.overlap_sms


def _row_chunks(T: int, n: int) -> list[tuple[int, int]]:
    """n row ranges of [0, T) on 256-row boundaries (fewer when T is small)."""
    step = max(256, (T + n - 1) // n + 255) // 256 * 256
    return [(a, min(a + step, T)) for a in range(0, T, step)]


def _gategrad_into(dy2, x2, layer, out=None, reserve: int = 0) -> torch.Tensor:
    in_f, off = layer.in_features, layer.in_col_offset
    if off:  # halo shard: zero inputs for the stored columns before the rank's own
        x2 = F.pad(x2[:, :in_f], (off, 0))
    if reserve:  # leave SMs to the all-reduce in flight so that it overlaps the GEMM
        _C.set_gategrad_sm_reserve(reserve)
    try:
        return _C.gategrad(dy2, x2, layer.candidate_types, layer._candidate_blocks(), layer.out_features,
                           off + in_f, layer.padded_in_features,
                           workspace=layer._gategrad_workspace(x2.device), out=out)
    finally:
        if reserve:
            _C.set_gategrad_sm_reserve(0)


def _gg_groupable(layers) -> bool:
    """Whether the gate gradients of gated Linears that share an input run as
    one grouped gate-gradient GEMM: two to four layers, the same candidate
    formats and padded width, each a multiple of 32 output rows."""
    l0 = layers[0]
    return 2 <= len(layers) <= 4 and all(
        l.candidate_types == l0.candidate_types and l.padded_in_features == l0.padded_in_features and
        l.out_features % 32 == 0 and not l.in_col_offset for l in layers)


def _gategrad_group_into(dy2, x2, layers, out=None, reserve: int = 0) -> torch.Tensor:
    """[G, K] gate gradients of `layers` (outputs side by side in dy2's
    columns) from one grouped gate-gradient GEMM."""
    l0 = layers[0]
    rows = [l.out_features for l in layers]
    need = _C.gategrad_grouped_workspace_bytes(sum(rows), l0.in_features, len(layers), l0.num_candidates)
    ws = getattr(l0, "_gws", None)
    if ws is None or ws.device != x2.device or ws.numel() < need:
        ws = torch.empty(max(need, 4), dtype=torch.uint8, device=x2.device)
        l0._gws = ws
    if reserve:
        _C.set_gategrad_sm_reserve(reserve)
    try:
        return _C.gategrad_grouped(dy2, x2, l0.candidate_types, [l._candidate_blocks() for l in layers], rows,
                                   l0.in_features, l0.padded_in_features, workspace=ws, out=out)
    finally:
        if reserve:
            _C.set_gategrad_sm_reserve(0)


def _group_rows_view(slots):
    """The bank-gradient rows `slots` as one [G, K] view when they are
    consecutive rows of one buffer, else None."""
    s0 = slots[0]
    if s0.dim() != 1 or s0.stride(0) != 1:
        return None
    base = s0._base if s0._base is not None else None
    if base is None or base.dim() != 2:
        return None
    ld = base.stride(0)
    for i, s in enumerate(slots):
        if s.numel() != s0.numel() or s.data_ptr() != s0.data_ptr() + i * ld * s0.element_size():
            return None
    return s0.as_strided((len(slots), s0.numel()), (ld, 1))


def _group_gategrad_to_slots(dy2, x2, layers, slots, reserve: int = 0) -> None:
    view = _group_rows_view(slots)
    if view is not None:
        _gategrad_group_into(dy2, x2, layers, out=view, reserve=reserve)
        return
    g = _gategrad_group_into(dy2, x2, layers, reserve=reserve)
    for i, s in enumerate(slots):
        s.copy_(g[i])


# Gate-gradient GEMMs deferred until the all-reduce of their module's input
# gradient is in flight (TP): (dY, X, layer, destination row of the bank's
# gradient buffer), or (dY, X, tuple of layers, list of their rows) for a
# grouped gate-gradient GEMM.  parallel._CopyToParallel.backward launches that
# all-reduce asynchronously and then runs these beside it; the gate bank's
# backward runs what is left, so every deferred GEMM precedes its reader.
_DEFERRED: list = []


def has_deferred_gategrads() -> bool:
    return bool(_DEFERRED)


def flush_deferred_gategrads(overlap_bytes: int = 0) -> None:
    """Run the deferred gate-gradient GEMMs in order.  The first ones, about
    as long as an all-reduce of `overlap_bytes` in flight, leave SMs to it."""
    from voodoo_quant.parallel import TP
    sms = _overlap_sms() if overlap_bytes else 0
    w = max(TP.world_size, 2)
    budget = overlap_bytes * 2.0 * (w - 1) / w / 450e9  # seconds at a ring bus bandwidth of 450 GB/s
    items = list(_DEFERRED)
    _DEFERRED.clear()
    for dy2, x2, layer, out in items:
        if isinstance(layer, tuple):
            _group_gategrad_to_slots(dy2, x2, layer, out, reserve=sms if budget > 0 else 0)
            budget -= 2.0 * x2.shape[0] * sum(l.out_features for l in layer) * layer[0].in_features / 1.2e15
            continue
        _gategrad_into(dy2, x2, layer, out=out, reserve=sms if budget > 0 else 0)
        budget -= 2.0 * x2.shape[0] * layer.out_features * layer.in_features / 1.2e15


def _defer_slot(layer) -> torch.Tensor | None:
    """The bank gradient row this layer's gate gradient goes to when it is
    deferred, else None."""
    bank = layer.__dict__.get("_bank_ref")
    if bank is None or not layer.__dict__.get("_defer_gategrad", False) or bank._dgrad is None:
        return None
    return bank._dgrad[layer._bank_index, :layer.num_candidates]


def _gated_linear_backward(ctx, dy: torch.Tensor):
    """dX = dY W_mix and d probs_k = <dY^T X, W_k>: the mixture's Jacobian,
    shared by the mixture forward and the routed (PTQR) forward."""
    layer = ctx.layer
    x2, probs = ctx.saved_tensors
    dy2 = _C._as_operand(dy.reshape(-1, layer.out_features))
    dx = dprobs = None
    pending = []
    if ctx.needs_input_grad[0]:
        w_mix = ctx.w_mix if ctx.w_mix is not None else layer._mix(probs)
        from voodoo_quant.parallel import sp_enabled
        if layer.reduce_input_grad and not sp_enabled():
            # column-parallel layer with a private input: sum the partial
            # dX over the TP ranks (chunk by chunk) while the rest of dX and
            # the gate-gradient GEMM run
            from voodoo_quant.parallel import tp_all_reduce_async
            T = dy2.shape[0]
            chunks = _row_chunks(T, INPUT_GRAD_CHUNKS) if INPUT_GRAD_CHUNKS > 1 else [(0, T)]
            dx = torch.empty(T, layer.in_features, dtype=torch.bfloat16, device=dy2.device)
            sms = _overlap_sms() if len(chunks) > 1 else 0
            try:
                for i, (a, b) in enumerate(chunks):
                    if i == 1 and sms:  # later chunks leave SMs to the all-reduces in flight
                        _C.set_gemm_sm_reserve(sms)
                    _C.linear_dx(dy2[a:b], w_mix, layer.in_features, out=dx[a:b])
                    pending.append(tp_all_reduce_async(dx[a:b], overlap=True))
            finally:
                if sms:
                    _C.set_gemm_sm_reserve(0)
        else:
            dx = _C.linear_dx(dy2, w_mix, layer.in_features)
    ctx.w_mix = None
    if ctx.needs_input_grad[1]:
        slot = None if pending else _defer_slot(layer)
        if slot is not None:  # runs beside the all-reduce of the module's input gradient
            _DEFERRED.append((dy2, x2, layer, slot))
        else:
            dprobs = _gategrad_into(dy2, x2, layer, reserve=_overlap_sms() if pending else 0).to(probs.dtype)
    for w in pending:
        w.wait()
    if dx is not None:
        dx = dx.to(ctx.x_dtype).reshape(ctx.x_shape)
    return dx, dprobs


class _GroupedGatedLinearFunction(Function):
    """Gated Linears that read the same input (q/k/v, gate/up) as ONE GEMM:
    each layer's mixture is written into its row range of one bf16 weight
    [sum N_i, Kin], so the forward is one GEMM into Y [T, sum N_i] and the
    input gradient one GEMM dX = dY W_cat (the sum over the layers happens
    inside the GEMM's reduction, not as separate dX tensors added up).  Each
    layer's gate gradient is its own gate-gradient GEMM over its column range
    of dY.  Values are those of the per-layer path: the same mixtures, the
    same products, fp32 accumulation (dX sums over sum N_i instead of adding
    bf16 partial results, which is closer to the exact sum)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, layers: tuple, *probs: torch.Tensor):
        in_f = layers[0].in_features
        x2 = _C._as_operand(x.reshape(-1, in_f))
        w_cat = _mix_group(layers, probs)
        y = _C.linear_fwd(x2, w_cat, w_cat.shape[0], in_f)
        ctx.layers = layers
        ctx.x_shape = x.shape
        ctx.x_dtype = x.dtype
        ctx.save_for_backward(x2, *probs)
        ctx.w_cat = w_cat if KEEP_MIXED_WEIGHT else None
        return y.to(x.dtype).reshape(*x.shape[:-1], w_cat.shape[0])

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        layers = ctx.layers
        x2, *probs = ctx.saved_tensors
        n_tot = sum(l.out_features for l in layers)
        dy2 = _C._as_operand(dy.reshape(-1, n_tot))
        dx = None
        if ctx.needs_input_grad[0]:
            w_cat = ctx.w_cat if ctx.w_cat is not None else _mix_group(layers, probs)
            dx = _C.linear_dx(dy2, w_cat, layers[0].in_features)
            dx = dx.to(ctx.x_dtype).reshape(ctx.x_shape)
        ctx.w_cat = None
        need = [ctx.needs_input_grad[2 + i] for i in range(len(layers))]
        if all(need) and _gg_groupable(layers):
            # every layer's gate gradient from one GEMM over all of dY's columns
            slots = [_defer_slot(l) for l in layers]
            if all(s is not None for s in slots):  # beside the all-reduce of the input gradient
                _DEFERRED.append((dy2, x2, tuple(layers), slots))
                return (dx, None, *([None] * len(layers)))
            if all(s is None for s in slots):
                g = _gategrad_group_into(dy2, x2, layers)
                return (dx, None, *[g[i].to(p.dtype) for i, p in enumerate(probs)])
        grads = []
        a = 0
        for i, layer in enumerate(layers):
            b = a + layer.out_features
            g = None
            if ctx.needs_input_grad[2 + i]:
                slot = _defer_slot(layer)
                if slot is not None:  # runs beside the all-reduce of the module's input gradient
                    _DEFERRED.append((dy2[:, a:b], x2, layer, slot))
                else:
                    g = _gategrad_into(dy2[:, a:b], x2, layer).to(probs[i].dtype)
            grads.append(g)
            a = b
        return (dx, None, *grads)


def _mix_group(layers, probs) -> torch.Tensor:
    """The layers' bf16 mixtures stacked by rows into one [sum N_i, ld] weight."""
    in_f = layers[0].in_features
    ld = (in_f + 7) // 8 * 8
    dev = layers[0]._cand_arena.device
    w = torch.empty(sum(l.out_features for l in layers), ld, dtype=torch.bfloat16, device=dev)
    a = 0
    for layer, p in zip(layers, probs):
        b = a + layer.out_features
        _C.mix(layer.candidate_types, layer._candidate_blocks(), p.to(dev), layer.out_features,
               layer.padded_in_features, in_f, out=w[a:b])
        a = b
    return w


def groupable(layers) -> bool:
    """Whether gated Linears can run as one grouped GEMM: same input width,
    no halo or row-parallel shard, not PTQR-routed, no in-backward dX sum."""
    if _PTQR_STATE.enabled or len(layers) < 2:
        return False
    l0 = layers[0]
    for l in layers:
        if not isinstance(l, MixedQuantLinear) or l.in_features != l0.in_features or l.in_col_offset or \
                l.reduce_input_grad or l._cand_arena.device != l0._cand_arena.device or l.out_features % 8:
            return False
        spec = l.shard_spec
        if spec is not None and spec.col_offset is not None:
            return False
    return True


def gated_linear_group(layers, x: torch.Tensor) -> torch.Tensor:
    """y = x [W_1; W_2; ...]^T for gated Linears sharing the input x (see
    ``_GroupedGatedLinearFunction``): [..., sum N_i], layer i's outputs in
    columns [sum_{j<i} N_j, sum_{j<=i} N_j)."""
    layers = tuple(layers)
    if x.device != layers[0]._cand_arena.device:
        x = x.to(layers[0]._cand_arena.device)
    probs = [l.get_probs().to(x.device) for l in layers]
    return _GroupedGatedLinearFunction.apply(x, layers, *probs)


class _RoutedGatedLinearFunction(Function):
    """PTQR forward y[t] = x[t] W_{k(t)}^T, one candidate per token (reference
    _RoutedMixedLinear, voodoo_quant/layers.py:366-428).

    Tokens are grouped by candidate (a stable sort of the routing) and one
    grouped tcgen05 GEMM multiplies each group with its candidate's bf16
    decode (the mixture kernel with a one-hot probability), reading the group
    offsets on the device; rows are scattered back.  The GEMM FLOPs equal
    one dense forward.  Backward is the mixture's
    straight-through Jacobian: dX = dY W_mix, d p_k = <dY^T X, W_k>.
    """

    @staticmethod
    def forward(ctx, x: torch.Tensor, probs: torch.Tensor, layer: "MixedQuantLinear", routing: torch.Tensor,
                reduce_out: bool = False):
        in_f, out_f = layer.in_features, layer.out_features
        x2 = _C._as_operand(x.reshape(-1, in_f))
        T = x2.shape[0]
        routing = routing.to(x2.device).reshape(-1)
        # one kernel: stable grouping order, its inverse (the scatter back
        # becomes a vectorised row gather) and the group offsets
        order, inv, group_off = _C.route_prep(routing, layer.num_candidates)
        xs = x2.index_select(0, order)
        one = torch.ones(1, dtype=torch.float32, device=x2.device)
        blocks = layer._candidate_blocks()
        ws = [layer._mix_of([qt], [blocks[k]], one) for k, qt in enumerate(layer.candidate_types)]
        if T > 128:  # one grouped GEMM; the group sizes stay on the device
            ys = _C.linear_fwd_grouped(xs, ws, out_f, in_f, group_off)
        else:
            ys = torch.empty(T, out_f, dtype=torch.bfloat16, device=x2.device)
            offs = group_off.tolist()
            for k in range(layer.num_candidates):
                a, b = offs[k], offs[k + 1]
                if b > a:
                    _C.linear_fwd(xs[a:b], ws[k], out_f, in_f, out=ys[a:b])
        y = ys.index_select(0, inv)
        if reduce_out:
            from voodoo_quant.parallel import all_reduce_
            all_reduce_(y)
        ctx.layer = layer
        ctx.x_shape = x.shape
        ctx.x_dtype = x.dtype
        ctx.save_for_backward(x2, probs)
        ctx.w_mix = None  # the backward mixes W_mix itself
        return y.to(x.dtype).reshape(*x.shape[:-1], out_f)

    @staticmethod
    def backward(ctx, dy: torch.Tensor):
        dx, dprobs = _gated_linear_backward(ctx, dy)
        return dx, dprobs, None, None, None


class _MixedWeightFunction(Function):
    """W_mix as a tensor (get_mixed_weight); backward g_k = <G, W_k>."""

    @staticmethod
    def forward(ctx, probs: torch.Tensor, layer: "_MixedQuantBase"):
        ctx.layer = layer
        w = layer._mix(probs)
        return w[:, :layer.in_features].to(layer.source_dtype)

    @staticmethod
    def backward(ctx, g: torch.Tensor):
        layer = ctx.layer
        gf = g.to(torch.float32)
        out = torch.empty(layer.num_candidates, dtype=torch.float32, device=g.device)
        off = layer.in_col_offset
        for k, (qt, qb) in enumerate(zip(layer.candidate_types, layer._candidate_blocks())):
            w = _C.dequant(qb, qt, layer.out_features, layer.padded_in_features)[:, off:off + layer.in_features]
            out[k] = (gf * w).sum()
        return out, None


class _GatedEmbeddingRowsFunction(Function):
    """Mixed rows of a vocabulary-scale embedding; only the touched rows are decoded."""

    @staticmethod
    def forward(ctx, probs: torch.Tensor, rows: torch.Tensor, layer: "MixedQuantEmbedding",
                routing: torch.Tensor | None = None):
        D = layer.embedding_dim
        if routing is None:
            blocks = layer._row_blocks(rows)
            w = _C.mix(layer.candidate_types, blocks, probs, rows.numel(), layer.padded_in_features, D)[:, :D]
        elif _STATIC_STATE.enabled:
            # PTQR without a host round trip: every row decoded by each
            # candidate, row i keeping candidate routing[i]'s (K decodes of
            # the batch's rows instead of one)
            one = torch.ones(1, dtype=torch.float32, device=rows.device)
            w = None
            for k, qt in enumerate(layer.candidate_types):
                wk = _C.mix([qt], layer._row_blocks(rows, only=k), one, rows.numel(), layer.padded_in_features,
                            D)[:, :D]
                sel = (routing == k).unsqueeze(1)
                w = torch.where(sel, wk, w if w is not None else torch.zeros_like(wk))
        else:
            # PTQR: row i keeps candidate routing[i]'s decoded row (reference :712-717)
            w = torch.empty(rows.numel(), D, dtype=torch.bfloat16, device=rows.device)
            one = torch.ones(1, dtype=torch.float32, device=rows.device)
            for k, qt in enumerate(layer.candidate_types):
                idx = torch.nonzero(routing == k, as_tuple=False).squeeze(1)
                if idx.numel() == 0:
                    continue
                blk = layer._row_blocks(rows.index_select(0, idx), only=k)
                w[idx] = _C.mix([qt], blk, one, idx.numel(), layer.padded_in_features, D)[:, :D]
        ctx.layer = layer
        ctx.save_for_backward(rows)
        return w.to(layer.source_dtype)

    @staticmethod
    def backward(ctx, g: torch.Tensor):
        layer = ctx.layer
        (rows,) = ctx.saved_tensors
        gf = g.to(torch.float32)
        blocks = layer._row_blocks(rows)
        out = torch.empty(layer.num_candidates, dtype=torch.float32, device=g.device)
        for k, (qt, qb) in enumerate(zip(layer.candidate_types, blocks)):
            w = _C.dequant(qb, qt, rows.numel(), layer.padded_in_features)[:, :layer.embedding_dim]
            out[k] = (gf * w).sum()
        return out, None, None, None


# --------------------------------------------------------------------------- modules
class _MixedQuantBase(nn.Module):
    """Candidate loading, gates and bookkeeping shared by Linear and Embedding."""

    def __init__(self, candidate_types: list[str], source_weight: torch.Tensor, out_features: int,
                 in_features: int, imatrix: torch.Tensor | None = None, device=None, lazy: bool = False,
                 tensor_name: str = "unknown", qbytes_device=None, shard_spec=None,
                 full_source_weight: torch.Tensor | None = None, candidate_bytes: dict | None = None,
                 candidate_bytes_local: bool = False):
        super().__init__()
        self.candidate_types = list(candidate_types)
        self.num_candidates = len(self.candidate_types)
        for qt in self.candidate_types:
            if qt not in GPU_FORMATS:
                get_quant_info(qt)  # unknown type -> ValueError, as in the reference
                raise ValueError(f"{qt} has no B200 decoder; supported candidates: {list(GPU_FORMATS)}")
        if self.num_candidates < 1 or self.num_candidates > 8:
            raise ValueError(f"{tensor_name}: 1..8 candidates supported, got {self.num_candidates}")
        self.out_features = out_features
        self.in_features = in_features
        self.lazy = lazy
        self._tensor_name = tensor_name
        self.shard_spec = shard_spec
        if shard_spec is not None and full_source_weight is None and candidate_bytes is None:
            raise ValueError(f"{tensor_name}: shard_spec requires full_source_weight "
                             "(the unsharded weight for candidate quantization/caching)")
        if device is None:
            device = source_weight.device
        self._device = torch.device(device)
        self.gates = nn.Parameter(torch.zeros(self.num_candidates, device=self._device))
        self.temperature = 1.0
        self.source_dtype = source_weight.dtype
        self.imatrix = imatrix.detach().to(torch.float32).cpu() if imatrix is not None else None

        full = full_source_weight if shard_spec is not None else source_weight
        full_in = full.shape[1] if full is not None else in_features
        self._full_padded_in_features = _padded(full_in)
        if candidate_bytes is None:
            candidate_bytes = self._load_or_quantize(full, imatrix)
        qbytes = [candidate_bytes[qt] for qt in self.candidate_types]
        rows = shard_spec.full_out if shard_spec is not None else out_features
        self.padded_in_features = self._full_padded_in_features
        # column of input 0 inside the stored blocks: nonzero only for a halo
        # shard (parallel.ShardSpec.halo), whose blocks start before its columns
        self.in_col_offset = shard_spec.in_col_offset if shard_spec is not None else 0
        if shard_spec is not None:
            if not candidate_bytes_local:  # full-tensor candidates: keep this rank's blocks
                qbytes = [shard_spec.slice_qbytes(qb, qt, self._full_padded_in_features)
                          for qb, qt in zip(qbytes, self.candidate_types)]
            rows = shard_spec.local_out
            self.padded_in_features = shard_spec.local_padded_in(self._full_padded_in_features,
                                                                 self.candidate_types)
        qdev = torch.device(qbytes_device) if qbytes_device is not None else None
        if qdev is None or (qdev.type == "cuda" and qdev.index is None):
            if source_weight.is_cuda:
                qdev = source_weight.device
            elif self._device.type == "cuda":
                qdev = self._device
            elif qdev is None:
                qdev = torch.device("cpu")
        self._qbytes_device = qdev
        arena, layout = pack_arena(self.candidate_types, qbytes, rows, self.padded_in_features, qdev,
                                   tensor_name)
        self.register_buffer("_cand_arena", arena, persistent=False)
        self._cand_layout = layout
        self._ws = None
        STORE.register(tensor_name, self)

    # ---- candidate cache (reference format) ----
    def _load_or_quantize(self, weight: torch.Tensor, imatrix: torch.Tensor | None) -> dict:
        weight = weight.detach().to("cpu").contiguous()
        padded_im = None
        if imatrix is not None:
            _, padded_im, _ = _pad_weight_and_imatrix(
                torch.empty(1, weight.shape[1], dtype=torch.float32), imatrix.detach().to(torch.float32).cpu())
        wh = _tensor_hash(weight)
        ih = _tensor_hash(padded_im) if imatrix is not None else "none"
        name = self._tensor_name
        found: dict[str, torch.Tensor] = {}
        names = [name]
        names.append(name.removeprefix("model.") if name.startswith("model.") else "model." + name)
        for nm in names:
            p = _combined_cache_path(nm, "lazy", wh, ih)
            if p.exists():
                combined = _load_cache_file(p, name)
                for qt in self.candidate_types:
                    if qt in combined and qt not in found:
                        found[qt] = combined[qt]
                break
        missing = []
        for qt in self.candidate_types:
            if qt in found:
                continue
            p = _candidate_cache_path(name, qt, "lazy", wh, ih)
            if p.exists():
                found[qt] = _load_cache_file(p, name)
            else:
                missing.append((qt, p))
        if missing:
            padded, pim, _ = _pad_weight_and_imatrix(weight.to(torch.float32), padded_im if imatrix is not None else None)

            def quantize_one(item):
                qt, p = item
                qb = quantize_tensor(padded, qt, pim)  # libggml, exactly as the reference
                _atomic_torch_save(qb.cpu(), p)
                return qt, qb

            # one thread per missing candidate, as the reference does
            # (_quantize_candidates_parallel, layers.py:1282-1340): libggml
            # runs outside the GIL under ctypes
            import concurrent.futures

            workers = int(os.environ.get("VOODOO_QUANT_WORKERS", min(8, os.cpu_count() or 2)))
            with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(workers, len(missing)))) as ex:
                for qt, qb in ex.map(quantize_one, missing):
                    found[qt] = qb
        return found

    # ---- candidate access ----
    def _candidate_blocks(self) -> list[torch.Tensor]:
        return arena_views(self._cand_arena, self._cand_layout)

    def __getattr__(self, name: str):
        if name.startswith("_qweight_") and name[9:].isdigit():
            k = int(name[9:])
            layout = self.__dict__.get("_cand_layout")
            if layout is not None and k < len(layout):
                return self._candidate_blocks()[k]
        if name.startswith("_w_") and name[3:].isdigit():
            k = int(name[3:])
            layout = self.__dict__.get("_cand_layout")
            if layout is not None and k < len(layout):
                # Decoded on demand (bit-exact); never stored.
                qb = self._candidate_blocks()[k]
                w = _C.dequant(qb, self.candidate_types[k], self.out_features, self.padded_in_features)
                off = self.__dict__.get("in_col_offset", 0)
                return w[:, off:off + self.in_features].to(self.source_dtype)
        return super().__getattr__(name)

    def _mix(self, probs: torch.Tensor) -> torch.Tensor:
        return self._mix_of(self.candidate_types, self._candidate_blocks(), probs.to(self._cand_arena.device))

    def _mix_of(self, types: list[str], blocks: list[torch.Tensor], probs: torch.Tensor) -> torch.Tensor:
        """bf16 W_mix [out, in] of the given candidates.  A halo shard mixes its
        stored blocks up to its last column and returns the column window of
        its inputs: a strided view whose base stays 16-byte aligned (the
        offset is a multiple of 8 columns)."""
        off = self.in_col_offset
        w = _C.mix(types, blocks, probs, self.out_features, self.padded_in_features, off + self.in_features)
        return w[:, off:off + self.in_features] if off else w

    def _gategrad_workspace(self, device: torch.device) -> torch.Tensor:
        need = _C.gategrad_workspace_bytes(self.out_features, self.in_features + self.in_col_offset,
                                           self.num_candidates)
        if self._ws is None or self._ws.device != device or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 4), dtype=torch.uint8, device=device)
        return self._ws

    # ---- gates ----
    def set_temperature(self, temperature: float):
        self.temperature = max(temperature, 1e-6)

    def soft_probs(self) -> torch.Tensor:
        return F.softmax(self.gates / self.temperature, dim=0)

    def get_probs(self) -> torch.Tensor:
        bank = self.__dict__.get("_bank_probs")
        if bank is not None:  # this step's probabilities from a GateBank
            return bank
        return self.soft_probs()

    def invalidate_candidate_cache(self):
        """No cross-step dequant cache exists on this path (candidates stay packed)."""

    def get_mixed_weight(self) -> torch.Tensor:
        return _MixedWeightFunction.apply(self.get_probs(), self)

    def effective_bytes(self) -> torch.Tensor:
        probs = self.soft_probs()
        out_eff = getattr(self, "_full_out_features", None) or self.out_features
        in_eff = getattr(self, "_full_in_features", None) or self.in_features
        n = in_eff * out_eff
        bpw = torch.tensor([bytes_per_weight(qt) for qt in self.candidate_types], dtype=probs.dtype,
                           device=probs.device)
        return (probs * bpw).sum() * n

    def get_assignment(self) -> str:
        return self.candidate_types[self.gates.argmax().item()]

    def get_assignment_prob(self) -> float:
        probs = self.soft_probs().detach()
        return probs[self.gates.argmax().item()].item()

    # ---- TP restriction after construction (reference :1395-1472) ----
    def _repack(self, qbytes: list[torch.Tensor], rows: int, padded: int) -> None:
        arena, layout = pack_arena(self.candidate_types, qbytes, rows, padded, self._cand_arena.device,
                                   self._tensor_name)
        self._cand_arena = arena
        self._cand_layout = layout

    def shard_rows(self, row_ranges: list[tuple[int, int]]) -> None:
        if self.__dict__.get("_full_out_features") is not None or self.__dict__.get("_full_in_features") is not None:
            raise RuntimeError(f"{self._tensor_name}: already row/col-sharded")
        shard_out = sum(e - s for s, e in row_ranges)
        if shard_out <= 0 or shard_out > self.out_features:
            raise ValueError(f"{self._tensor_name}: invalid row ranges {row_ranges} "
                             f"for out_features={self.out_features}")
        new = []
        for qb in self._candidate_blocks():
            q2 = qb.reshape(self.out_features, -1)
            new.append(torch.cat([q2[s:e] for s, e in row_ranges], dim=0).reshape(-1))
        self._repack(new, shard_out, self.padded_in_features)
        self._full_out_features = self.out_features
        self.out_features = shard_out

    def shard_cols(self, col_range: tuple[int, int]) -> None:
        if self.__dict__.get("_full_out_features") is not None or self.__dict__.get("_full_in_features") is not None:
            raise RuntimeError(f"{self._tensor_name}: already row/col-sharded")
        s, e = col_range
        if s < 0 or e > self.in_features or e <= s:
            raise ValueError(f"{self._tensor_name}: invalid column range {col_range} "
                             f"for in_features={self.in_features}")
        new = []
        for qt, qb in zip(self.candidate_types, self._candidate_blocks()):
            info = get_quant_info(qt)
            if s % 256 or (e - s) % 256:
                raise ValueError(f"{self._tensor_name}: column range {col_range} is not "
                                 f"{info.block_size}-block aligned for {qt}")
            nbpr = self.padded_in_features // info.block_size
            q3 = qb.view(self.out_features, nbpr, info.block_bytes)[:, s // info.block_size:e // info.block_size]
            new.append(q3.reshape(-1))
        self._repack(new, self.out_features, e - s)
        self._full_in_features = self.in_features
        self.in_features = e - s
        self.padded_in_features = e - s


class MixedQuantLinear(_MixedQuantBase):
    """Linear layer whose weight is the softmax mixture of K packed candidates."""

    def __init__(self, in_features: int, out_features: int, candidate_types: list[str],
                 source_weight: torch.Tensor, imatrix: torch.Tensor | None = None, device=None,
                 lazy: bool = False, tensor_name: str = "unknown", qbytes_device=None, shard_spec=None,
                 full_source_weight: torch.Tensor | None = None, candidate_bytes: dict | None = None,
                 candidate_bytes_local: bool = False):
        super().__init__(candidate_types=candidate_types, source_weight=source_weight,
                         out_features=out_features, in_features=in_features, imatrix=imatrix, device=device,
                         lazy=lazy, tensor_name=tensor_name, qbytes_device=qbytes_device,
                         shard_spec=shard_spec, full_source_weight=full_source_weight,
                         candidate_bytes=candidate_bytes, candidate_bytes_local=candidate_bytes_local)
        if shard_spec is not None and shard_spec.vocab_start is not None:
            self.tp_vocab_start = shard_spec.vocab_start
            self.tp_vocab_end = shard_spec.vocab_start + out_features
        # Column-parallel layer whose input feeds no other TP shard: sum its dX
        # over the ranks inside the backward, overlapped with the gate-gradient
        # GEMM (instead of entering the input through parallel.tp_copy_to_parallel).
        self.reduce_input_grad = False

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        spec = self.shard_spec
        if x.device != self._cand_arena.device:
            x = x.to(self._cand_arena.device)
        if _PTQR_STATE.enabled:
            probs = self.get_probs().to(x.device)
            n = x.numel() // x.shape[-1]
            bank = self.__dict__.get("_bank_ref")
            routing = bank.routing(self, n) if bank is not None else _sample_token_routing(probs, n)
            # row-parallel: the partial outputs are summed over the TP ranks in
            # place (sequence parallelism: by the block's reduce-scatter)
            from voodoo_quant.parallel import sp_enabled
            reduce_out = spec is not None and spec.col_offset is not None and not sp_enabled()
            return _RoutedGatedLinearFunction.apply(x, probs, self, routing, reduce_out)
        from voodoo_quant.parallel import sp_enabled
        if spec is not None and spec.col_offset is not None and not sp_enabled():
            from voodoo_quant.parallel import nccl_row_reducer
            # the output sum over the TP ranks happens inside the forward (an
            # in-place NCCL all-reduce of the fresh GEMM output); its backward
            # is the identity, so the gradients are the local ones
            red = nccl_row_reducer()
            return _GatedLinearFunction.apply(x, self.get_probs().to(x.device), self, red)
        return _GatedLinearFunction.apply(x, self.get_probs().to(x.device), self)


class MixedQuantEmbedding(_MixedQuantBase):
    """Embedding whose table is the softmax mixture of K packed candidates."""

    def __init__(self, num_embeddings: int, embedding_dim: int, candidate_types: list[str],
                 source_weight: torch.Tensor, imatrix: torch.Tensor | None = None, device=None,
                 lazy: bool = False, tensor_name: str = "unknown", qbytes_device=None, shard_spec=None,
                 full_source_weight: torch.Tensor | None = None, candidate_bytes: dict | None = None,
                 candidate_bytes_local: bool = False):
        super().__init__(candidate_types=candidate_types, source_weight=source_weight,
                         out_features=num_embeddings, in_features=embedding_dim, imatrix=imatrix,
                         device=device, lazy=lazy, tensor_name=tensor_name, qbytes_device=qbytes_device,
                         shard_spec=shard_spec, full_source_weight=full_source_weight,
                         candidate_bytes=candidate_bytes, candidate_bytes_local=candidate_bytes_local)
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        if shard_spec is not None and shard_spec.vocab_start is not None:
            self.tp_vocab_start = shard_spec.vocab_start
            self.tp_vocab_end = shard_spec.vocab_start + num_embeddings

    def _row_blocks(self, rows: torch.Tensor, only: int | None = None) -> list[torch.Tensor]:
        out = []
        for k, (qt, qb) in enumerate(zip(self.candidate_types, self._candidate_blocks())):
            if only is not None and k != only:
                continue
            info = get_quant_info(qt)
            nbpr = self.padded_in_features // info.block_size
            out.append(qb.view(self.num_embeddings, nbpr * info.block_bytes).index_select(0, rows).reshape(-1))
        return out

    def _embedding_lookup(self, ids: torch.Tensor) -> torch.Tensor:
        dev = self._cand_arena.device
        probs = self.get_probs().to(dev)
        if _STATIC_STATE.enabled:  # one row per token: no host round trip
            rows = ids.reshape(-1).to(dev)
            if _PTQR_STATE.enabled:  # one candidate per table row, looked up per token
                routing = _sample_token_routing(probs, self.num_embeddings).index_select(0, rows)
                mixed = _GatedEmbeddingRowsFunction.apply(probs, rows, self, routing)
            else:
                mixed = _GatedEmbeddingRowsFunction.apply(probs, rows, self)
            return mixed.reshape(*ids.shape, self.embedding_dim)
        rows, inverse = torch.unique(ids.reshape(-1).to(dev), return_inverse=True)
        if _PTQR_STATE.enabled:  # one candidate per (unique) row, reference layers.py:1810-1813
            routing = _sample_token_routing(probs, rows.shape[0])
            mixed = _GatedEmbeddingRowsFunction.apply(probs, rows, self, routing)
        else:
            mixed = _GatedEmbeddingRowsFunction.apply(probs, rows, self)
        return mixed[inverse].reshape(*ids.shape, self.embedding_dim)

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        spec = self.shard_spec
        if spec is not None and spec.vocab_start is not None:
            from voodoo_quant.parallel import sp_enabled, tp_all_reduce_sum_
            v0, v1 = self.tp_vocab_start, self.tp_vocab_end
            ids = input.to(self._cand_arena.device)
            in_shard = (ids >= v0) & (ids < v1)
            if _STATIC_STATE.enabled:
                # every token at a clamped row, other shards' rows zeroed; their
                # gradient is then zero, so the gate dots are this shard's alone
                local = (ids - v0).clamp(0, self.num_embeddings - 1)
                emb = self._embedding_lookup(local) * in_shard.unsqueeze(-1).to(self.source_dtype)
                return emb if sp_enabled() else tp_all_reduce_sum_(emb)
            # Only this shard's tokens are looked up: clamping the others to
            # one row would funnel most of the batch's gradient into a single
            # index of the lookup's backward.
            emb_in = self._embedding_lookup(ids[in_shard] - v0)
            emb = emb_in.new_zeros(*ids.shape, self.embedding_dim)
            emb[in_shard] = emb_in
            return emb if sp_enabled() else tp_all_reduce_sum_(emb)
        return self._embedding_lookup(input)


# --------------------------------------------------------------------------- walkers
from voodoo_quant.arch.base import DEFAULT_ATTENTION_SEGMENTS as _DEFAULT_SEGMENTS  # noqa: E402

_ATTENTION_SEGMENTS: frozenset = _DEFAULT_SEGMENTS


def resolve_candidate_types(tensor_name: str, base_candidates: list[str],
                            attention_candidates: list[str] | None = None,
                            non_attention_candidates: list[str] | None = None) -> list[str]:
    """Per-role candidate menu (reference voodoo_quant/layers.py:1870-1905)."""
    if attention_candidates is None and non_attention_candidates is None:
        return list(base_candidates)
    is_attn = any(seg in _ATTENTION_SEGMENTS for seg in tensor_name.split("."))
    group = attention_candidates if (is_attn and attention_candidates) else non_attention_candidates
    if not group:
        return list(base_candidates)
    return [qt for qt in group if qt in set(base_candidates)]


def _provided(provider, name: str, weight: torch.Tensor, types: list[str], spec=None):
    """Packed candidates from ``provider``: of the whole (256-padded) weight,
    or, for a TP shard, of only the rank's rows and stored block columns
    (``ShardSpec.local_block_weight``), which the layer then takes as they are."""
    if provider is None:
        return None
    if spec is not None:
        return provider(name, spec.local_block_weight(weight.detach()), types)
    padded, _, _ = _pad_weight_and_imatrix(weight.detach(), None)
    return provider(name, padded, types)


def replace_linear_with_mixed_quant(module: nn.Module, candidate_types: list[str] | None, prefix: str = "",
                                    target_names: Optional[set[str]] = None,
                                    skip_names: Optional[set[str]] = None,
                                    imatrix_dict: Optional[dict[str, torch.Tensor]] = None, device=None,
                                    lazy: bool = False, attention_candidates: Optional[list[str]] = None,
                                    non_attention_candidates: Optional[list[str]] = None,
                                    qbytes_device=None, candidate_provider=None) -> dict[str, _MixedQuantBase]:
    """Recursively replace selected nn.Linear children (reference :1908-2066).

    ``candidate_provider(name, weight, types) -> {qtype: uint8 blocks}``,
    when given, supplies packed candidates instead of the on-disk cache /
    libggml: of the whole tensor (padded to a multiple of 256 columns), or,
    for a TP-sharded child, of the rank's part only
    (``ShardSpec.local_block_weight``), which the packed formats allow
    because they are block-local.
    """
    if candidate_types is None:
        candidate_types = list(GPU_FORMATS)
    skip_names = skip_names or set()
    imatrix_dict = imatrix_dict or {}
    replaced: dict[str, _MixedQuantBase] = {}
    for name, child in list(module.named_children()):
        full_name = f"{prefix}.{name}" if prefix else name
        if name in skip_names:
            continue
        if isinstance(child, nn.Linear):
            if child.bias is not None:
                raise NotImplementedError(f"MixedQuantLinear does not support bias but {full_name} has one")
            if target_names is not None and name not in target_names:
                continue
            im = imatrix_dict.get(full_name, imatrix_dict.get(full_name + ".weight"))
            types = resolve_candidate_types(full_name, candidate_types, attention_candidates, non_attention_candidates)
            full_w = getattr(child, "tp_full_weight", None)
            spec = getattr(child, "tp_shard_spec", None)
            local = candidate_provider is not None and spec is not None and full_w is not None
            new = MixedQuantLinear(
                in_features=child.in_features, out_features=child.out_features, candidate_types=types,
                source_weight=child.weight.data, imatrix=im, device=device, lazy=lazy, tensor_name=full_name,
                qbytes_device=qbytes_device, shard_spec=spec, full_source_weight=full_w,
                candidate_bytes=_provided(candidate_provider, full_name,
                                          full_w if full_w is not None else child.weight.data, types,
                                          spec if local else None),
                candidate_bytes_local=local)
            if getattr(child, "_tp_input_copy", False):
                # the sharded child summed its input gradient over the ranks
                # through a pre-hook; the gated layer does it inside its backward
                from voodoo_quant.parallel import TP
                new.reduce_input_grad = TP.exact_input_grad
            setattr(module, name, new)
            replaced[full_name] = new
        else:
            replaced.update(replace_linear_with_mixed_quant(
                child, candidate_types, full_name, target_names, skip_names, imatrix_dict, device, lazy,
                attention_candidates, non_attention_candidates, qbytes_device, candidate_provider))
    return replaced


def replace_embedding_with_mixed_quant(module: nn.Module, candidate_types: list[str] | None, prefix: str = "",
                                       skip_names: Optional[set[str]] = None,
                                       imatrix_dict: Optional[dict[str, torch.Tensor]] = None, device=None,
                                       lazy: bool = False, qbytes_device=None,
                                       attention_candidates: Optional[list[str]] = None,
                                       non_attention_candidates: Optional[list[str]] = None,
                                       candidate_provider=None) -> dict[str, MixedQuantEmbedding]:
    """Recursively replace nn.Embedding children (reference :2086-2153)."""
    if candidate_types is None:
        candidate_types = list(GPU_FORMATS)
    skip_names = skip_names or set()
    imatrix_dict = imatrix_dict or {}
    replaced: dict[str, MixedQuantEmbedding] = {}
    for name, child in list(module.named_children()):
        full_name = f"{prefix}.{name}" if prefix else name
        if name in skip_names:
            continue
        if isinstance(child, nn.Embedding):
            im = imatrix_dict.get(full_name, imatrix_dict.get(full_name + ".weight"))
            types = resolve_candidate_types(full_name, candidate_types, attention_candidates, non_attention_candidates)
            full_w = getattr(child, "tp_full_weight", None)
            spec = getattr(child, "tp_shard_spec", None)
            local = candidate_provider is not None and spec is not None and full_w is not None
            new = MixedQuantEmbedding(
                num_embeddings=child.num_embeddings, embedding_dim=child.embedding_dim, candidate_types=types,
                source_weight=child.weight.data, imatrix=im, device=device, lazy=lazy, tensor_name=full_name,
                qbytes_device=qbytes_device, shard_spec=spec, full_source_weight=full_w,
                candidate_bytes=_provided(candidate_provider, full_name,
                                          full_w if full_w is not None else child.weight.data, types,
                                          spec if local else None),
                candidate_bytes_local=local)
            setattr(module, name, new)
            replaced[full_name] = new
        else:
            replaced.update(replace_embedding_with_mixed_quant(
                child, candidate_types, full_name, skip_names, imatrix_dict, device, lazy, qbytes_device,
                attention_candidates, non_attention_candidates, candidate_provider))
    return replaced


class GateBank:
    """All gated layers' softmax(g / tau) in one batched computation per step.

    ``probs()`` pads every layer's gates into one [L, Kmax] matrix (-inf in
    the padding), takes one softmax, and hands each layer a row view as the
    probabilities its forward uses until ``release()``; ``effective_bytes``
    is the same sum as ``total_effective_bytes`` from that matrix.  A step
    then launches a handful of kernels for the gates instead of several per
    layer for the forward and again for the size term.  Gradients reach each
    layer's ``gates`` parameter through the padding as usual.
    """

    def __init__(self, replaced: dict[str, "_MixedQuantBase"]):
        self.layers = list(replaced.values())
        if not self.layers:
            raise ValueError("GateBank needs at least one gated layer")
        dev = self.layers[0].gates.device
        self.kmax = max(l.num_candidates for l in self.layers)
        L = len(self.layers)
        idx, mask = [], torch.zeros(L, self.kmax, dtype=torch.bool)
        bpwn = torch.zeros(L, self.kmax, dtype=torch.float64)
        for i, l in enumerate(self.layers):
            mask[i, :l.num_candidates] = True
            out_eff = l.__dict__.get("_full_out_features") or l.out_features
            in_eff = l.__dict__.get("_full_in_features") or l.in_features
            for k, qt in enumerate(l.candidate_types):
                bpwn[i, k] = bytes_per_weight(qt) * in_eff * out_eff
            idx.extend(i * self.kmax + k for k in range(l.num_candidates))
        self.flat_index = torch.tensor(idx, dtype=torch.long, device=dev)
        self.valid = mask.to(dev)
        self.bpwn = bpwn.to(torch.float32).to(dev)
        self._p = None
        self._routes = {}
        self._dgrad = None
        # the temperature as a device scalar (set_temperature); None = each
        # layer's own Python float
        self.tau_t: torch.Tensor | None = None
        # gate gradients of layers marked _defer_gategrad are written into a
        # [L, Kmax] buffer (TP: they run beside an all-reduce) and reach the
        # gates through the tap below
        self.defer = any(l.__dict__.get("_defer_gategrad", False) for l in self.layers)

    def set_temperature(self, tau: float) -> None:
        """Every layer's temperature, also held in a device scalar that
        ``probs()`` divides by, so a recorded CUDA graph of the step reads
        the current value when it is replayed (a Python float would be frozen
        into it).  The division is the same float32 operation either way."""
        for l in self.layers:
            l.set_temperature(tau)
        t = max(float(tau), 1e-6)
        if self.tau_t is None:
            self.tau_t = torch.full((), t, dtype=torch.float32, device=self.layers[0].gates.device)
        else:
            self.tau_t.fill_(t)

    def probs(self) -> torch.Tensor:
        if self.tau_t is not None:
            g = torch.cat([l.gates for l in self.layers]) / self.tau_t
        else:
            g = torch.cat([l.gates / l.temperature for l in self.layers])
        padded = torch.full((len(self.layers) * self.kmax,), float("-inf"), dtype=g.dtype, device=g.device)
        padded = padded.index_put((self.flat_index,), g)
        p = torch.softmax(padded.view(len(self.layers), self.kmax), dim=1)
        pl = p
        _DEFERRED.clear()  # nothing left from a backward that did not finish
        if self.defer and torch.is_grad_enabled() and p.requires_grad:
            self._dgrad = torch.zeros(p.shape, dtype=torch.float32, device=p.device)
            pl = _BankTap.apply(p, self)
        else:
            self._dgrad = None
        for i, l in enumerate(self.layers):
            l._bank_probs = pl[i, :l.num_candidates]
            l._bank_ref = self
            l._bank_index = i
        self._p = p
        self._routes = {}
        return p

    def routing(self, layer: "_MixedQuantBase", num_tokens: int) -> torch.Tensor:
        """This step's PTQR routing of `layer` over `num_tokens` tokens.

        The first request for a token count samples every layer at once: the
        reference's Gumbel-argmax per layer and token (_sample_token_routing)
        as one [L, Kmax, T] draw, with the padding candidates never chosen.
        """
        r = self._routes.get(num_tokens)
        if r is None:
            p = self._p.detach()
            u = torch.rand(p.shape[0], p.shape[1], num_tokens, device=p.device)
            gumbel = -torch.log((-torch.log(u.clamp_min(1e-9))).clamp_min(1e-9))
            scores = torch.log(p.clamp_min(1e-9)).unsqueeze(2) + gumbel
            scores.masked_fill_(~self.valid.unsqueeze(2), float("-inf"))
            r = scores.argmax(dim=1).to(torch.uint8)
            self._routes[num_tokens] = r
        return r[layer._bank_index]

    def effective_bytes(self) -> torch.Tensor:
        if self._p is None:
            raise RuntimeError("GateBank.probs() must run first in this step")
        return (self._p * self.bpwn).sum()

    def release(self) -> None:
        for l in self.layers:
            l._bank_probs = None
            l._bank_ref = None
        self._p = None
        self._routes = {}
        self._dgrad = None


class _BankTap(Function):
    """Identity on the bank's probabilities; its backward adds the gate
    gradients that deferred layers wrote into the bank's buffer (after
    running any deferred GEMM still queued)."""

    @staticmethod
    def forward(ctx, p: torch.Tensor, bank: GateBank) -> torch.Tensor:
        ctx.bank = bank
        ctx.dgrad = bank._dgrad
        return p.view_as(p)

    @staticmethod
    def backward(ctx, g: torch.Tensor):
        flush_deferred_gategrads()
        return g + ctx.dgrad.to(g.dtype), None


def total_effective_bytes(replaced: dict[str, _MixedQuantBase]) -> torch.Tensor:
    total = None
    for layer in replaced.values():
        eb = layer.effective_bytes()
        total = eb if total is None else total + eb.to(total.device)
    return total if total is not None else torch.tensor(0.0)
