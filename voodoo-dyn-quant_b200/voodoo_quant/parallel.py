"""Tensor parallelism for the gated-candidate step (drop-in for voodoo_quant/parallel.py).

Same mechanism/policy split as the reference (voodoo_quant/parallel.py):
``ShardSpec`` + ``_shard_child`` + ``Column/RowParallelLinear`` /
``VocabParallelEmbedding`` are the mechanism; arch adapters
(:mod:`voodoo_quant.arch`) are the policy.  One process per GPU, NCCL over
NVLink/NVSwitch for the collectives (gloo on CPU for tests).

Differences from the reference, each for a reason:

* Exact input gradients.  The reference's column-parallel layers do no
  communication in backward (parallel.py:309-331), so the summed gate
  gradients of stacked blocks are inexact under TP.  Here every
  column-parallel input group (attention q/k/v, MLP gate/up) is entered
  through ``tp_copy_to_parallel`` -- identity forward, all-reduce of dX in
  backward (Megatron's "f" operator) -- installed once per group by the
  adapter.  ``TP.exact_input_grad = False`` restores the reference behaviour.
* Uneven, block-aligned shards.  ``block_aligned_split`` splits a dimension
  into 256-element units as evenly as possible (e.g. 25600 over 8 ranks =
  13,13,13,13,12,12,12,12 units), which the reference refuses
  (parallel.py:285-299).
* Halo shards for head-aligned row-parallel inputs.  Where a rank's whole
  attention heads end inside a 256-weight block (a 32B-shape o_proj at TP-8:
  5 heads x 128 = 640 columns), the reference refuses the split
  (parallel.py:266-272) and a block-aligned split would break heads and
  their GQA groups.  ``ShardSpec(halo=True)`` keeps the rank's exact columns
  but stores the packed blocks that cover them (768 columns); the gated
  layer multiplies through the column window of its mixed weight, and its
  gate gradient sees zero inputs outside the window, so the rank sums stay
  exact (a block two ranks share is counted once, split by columns).
* ``tp_init`` only binds a CUDA device when CUDA is available, so the gloo
  path runs on CPU-only hosts (the reference calls ``torch.cuda.set_device``
  unconditionally, parallel.py:71).
* One flat all-reduce for all gate gradients (``all_reduce_gate_grads``)
  instead of one call per tensor (trainer.py:434-444).
"""

from __future__ import annotations

import contextlib
import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F
from torch.autograd import Function

UNIT = 256  # super-block width: every TP split of an input dimension is a multiple


class _TPState:
    enabled = False
    rank = 0
    world_size = 1
    local_rank = 0
    group = None
    device: torch.device | None = None
    exact_input_grad = True
    # second communicator for the input-gradient all-reduces that run beside
    # gate-gradient GEMMs, limited to `overlap_sms` CTAs (the SMs the GEMMs
    # leave free); None = those all-reduces use `group`
    overlap_group = None
    overlap_sms = 0
    # the communicator forward collectives use inside collectives_on(); None = group
    forward_override = None
    # sequence parallelism (enable_sequence_parallel): between the blocks the
    # hidden state is a [tokens / N, hidden] shard of consecutive tokens;
    # all-gather before the column-parallel inputs, reduce-scatter after the
    # row-parallel outputs (instead of all-reducing replicated activations)
    sequence_parallel = False
    # row-parallel outputs returned as partial sums for the caller to reduce
    # (deferred_row_sums(): the step that interleaves teacher layers with the
    # student's forward all-reduces)
    defer_row_sums = False


TP = _TPState()


def _fwd_group():
    return TP.forward_override if TP.forward_override is not None else TP.group


@contextlib.contextmanager
def collectives_on(group):
    """Forward-pass collectives issued inside the block (row-parallel sums,
    vocabulary-parallel lookups) go to ``group`` instead of the TP group; a
    model run on another stream beside the main one uses its own
    communicator, so the two streams' collectives never interleave on one."""
    prev = TP.forward_override
    TP.forward_override = group
    try:
        yield
    finally:
        TP.forward_override = prev


def tp_init(backend: str = "nccl", timeout_min: int = 240) -> bool:
    """Initialise TP from torchrun's env (WORLD_SIZE > 1 and RANK set)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1 or "RANK" not in os.environ:
        return False
    rank = int(os.environ["RANK"])
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local_rank)
    if not dist.is_initialized():
        kw = {}
        if backend == "nccl" and torch.cuda.is_available():
            kw["device_id"] = torch.device("cuda", local_rank)
        dist.init_process_group(backend=backend, init_method="env://", rank=rank, world_size=world,
                                timeout=timedelta(minutes=timeout_min), **kw)
    _adopt_group(local_rank)
    return True


def _adopt_group(local_rank: int = 0) -> None:
    TP.enabled = dist.get_world_size() > 1
    TP.rank = dist.get_rank()
    TP.world_size = dist.get_world_size()
    TP.local_rank = local_rank
    TP.group = dist.group.WORLD
    TP.device = torch.device("cuda", local_rank) if dist.get_backend() == "nccl" else torch.device("cpu")


def adopt_process_group(local_rank: int = 0) -> None:
    """Use an already-initialised default process group for TP (tests, embedding)."""
    _adopt_group(local_rank)


def init_tp(backend: str | None = None, timeout_min: int = 240) -> tuple[int, int]:
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() and dist.is_nccl_available() else "gloo"
    tp_init(backend=backend, timeout_min=timeout_min)
    return TP.rank, TP.world_size


def tp_finalize() -> None:
    if TP.enabled and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    TP.enabled = False
    TP.rank, TP.world_size = 0, 1


def reset_tp() -> None:
    TP.enabled = False
    TP.rank, TP.world_size, TP.local_rank = 0, 1, 0
    TP.group = None
    TP.device = None
    TP.overlap_group = None
    TP.overlap_sms = 0
    TP.forward_override = None
    TP.sequence_parallel = False
    TP.defer_row_sums = False


def teacher_subgroups(t: int):
    """Split the TP ranks into world / t groups of t consecutive ranks, one
    communicator each, for a teacher sharded t ways that runs on 1 / (world / t)
    of the batch per group.  Collective: every rank calls it with the same t.
    Returns (this rank's group, its index, the rank's index within it)."""
    W, r = TP.world_size, TP.rank
    if t < 1 or W % t:
        raise ValueError(f"teacher TP degree {t} does not divide the TP world size {W}")
    mine = None
    for g in range(W // t):
        grp = dist.new_group(ranks=list(range(g * t, (g + 1) * t)), backend=dist.get_backend(TP.group))
        if g == r // t:
            mine = grp
    return mine, r // t, r % t


@contextlib.contextmanager
def as_tp(rank: int, world: int, group):
    """Inside the block this process is rank ``rank`` of a TP group of
    ``world`` ranks on ``group`` (a sub-group of the TP ranks): what the arch
    adapters read when they shard a model (``tp_patch_model``)."""
    saved = (TP.rank, TP.world_size, TP.group)
    TP.rank, TP.world_size, TP.group = rank, world, group
    try:
        yield
    finally:
        TP.rank, TP.world_size, TP.group = saved


def redistribute_vocab_shards(local: torch.Tensor, t: int, group=None) -> torch.Tensor:
    """Teacher logits from the (batch-slice, t-way vocabulary) layout to the
    student's (whole batch, world-way vocabulary) layout, in one all-to-all.

    ``local`` is this rank's [b, S, V / t]: the rows of batch slice g = rank // t
    (b = B / G, G = world / t groups) and vocabulary part h = rank % t.  Student
    rank r needs every row over columns [r V / world, (r + 1) V / world), which
    lie in teacher part r // G; so rank (g, h) sends its G column chunks to
    student ranks h G ... h G + G - 1 and each rank receives one [b, S, V / world]
    chunk from rank (g', r // G) of every group g'.  Returns [B, S, V / world]."""
    W, r = TP.world_size, TP.rank
    G = W // t
    h = r % t
    b, S, Vt = local.shape
    if Vt % G:
        raise ValueError(f"teacher vocabulary part {Vt} does not split into {G} student slices")
    Vw = Vt // G
    n = b * S * Vw
    send = local.reshape(b * S, G, Vw).permute(1, 0, 2).contiguous()  # chunk j -> student rank h G + j
    in_splits, out_splits = [0] * W, [0] * W
    for j in range(G):
        in_splits[h * G + j] = n
    for g2 in range(G):
        out_splits[g2 * t + r // G] = n
    # all-to-all moves bytes only: 16-bit logits travel as float16 bit patterns
    # (every backend carries float16)
    wire = send.view(torch.float16) if send.dtype == torch.bfloat16 else send
    out = torch.empty(G * n, dtype=wire.dtype, device=local.device)
    dist.all_to_all_single(out, wire.reshape(-1), out_splits, in_splits, group=group)
    if send.dtype == torch.bfloat16:
        out = out.view(torch.bfloat16)
    return out.view(G * b, S, Vw)


def enable_input_grad_overlap(sms: int) -> bool:
    """Run input-gradient all-reduces beside the gate-gradient GEMMs.

    Collective: every rank calls it with the same `sms`.  Creates a second
    communicator whose collectives use at most `sms` CTAs (NCCL maxCTAs) and
    makes the GEMMs that run beside them leave that many SMs free; the
    forward's all-reduces keep the default communicator and all its
    channels.  `sms` <= 0 turns the overlap off.  Returns whether it is on.
    """
    if not TP.enabled or sms <= 0:
        TP.overlap_group, TP.overlap_sms = None, 0
        return False
    ranks = list(range(TP.world_size))
    if dist.get_backend(TP.group) == "nccl":
        opts = dist.ProcessGroupNCCL.Options()
        opts.config.max_ctas = int(sms)
        opts.config.min_ctas = min(int(sms), 8)
        opts.is_high_priority_stream = True
        TP.overlap_group = dist.new_group(ranks=ranks, backend="nccl", pg_options=opts)
    else:
        TP.overlap_group = dist.new_group(ranks=ranks, backend=dist.get_backend(TP.group))
    TP.overlap_sms = int(sms)
    return True


@contextlib.contextmanager
def deferred_row_sums(on: bool = True):
    """Inside the block, a row-parallel gated Linear starts the all-reduce of
    its output in place without waiting for it (``take_row_sums`` hands the
    caller the handles, which it waits on before reading the outputs)."""
    prev = TP.defer_row_sums
    TP.defer_row_sums = bool(on) and TP.enabled
    try:
        yield
    finally:
        TP.defer_row_sums = prev


_ROW_SUMS: list = []


def take_row_sums() -> list:
    """The handles of the row-parallel sums started since the last call."""
    works = list(_ROW_SUMS)
    _ROW_SUMS.clear()
    return works


def sp_enabled() -> bool:
    """Whether the TP hidden states between blocks are token shards."""
    return TP.enabled and TP.sequence_parallel


def enable_sequence_parallel(enable: bool = True) -> bool:
    """Sequence parallelism for the models that ``use_sequence_parallel``
    patched (voodoo_quant.fused_blocks): the residual stream, the RMSNorms
    and the residual adds then run on each rank's [tokens / N, hidden] shard;
    each attention / MLP block all-gathers its normalised input and
    reduce-scatters its row-parallel output, which moves the same bytes as
    the all-reduce it replaces.  Row-parallel layers and vocabulary-parallel
    embeddings then return their partial sums.  Returns whether it is on."""
    TP.sequence_parallel = bool(enable) and TP.enabled
    return TP.sequence_parallel


def _group_size(group) -> int:
    return dist.get_world_size(group) if group is not None else TP.world_size


class _SPGather(Function):
    """Token shard [n, H] -> all tokens [N n, H] (rank order) over the forward
    group; backward: reduce-scatter of the gradient, beside which the gate-
    gradient GEMMs deferred by the block it feeds run (on the overlap
    communicator, as for the f operator's all-reduce)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor) -> torch.Tensor:
        group = _fwd_group()
        W = _group_size(group)
        ctx.group = group
        x = x.contiguous()
        out = torch.empty((W * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        from voodoo_quant import layers

        g = g.contiguous()
        W = _group_size(ctx.group)
        out = torch.empty((g.shape[0] // W,) + tuple(g.shape[1:]), dtype=g.dtype, device=g.device)
        if layers.has_deferred_gategrads() and ctx.group is TP.group:
            grp = TP.overlap_group if TP.overlap_group is not None else TP.group
            work = dist.reduce_scatter_tensor(out, g, group=grp, async_op=True)
            layers.flush_deferred_gategrads(overlap_bytes=g.numel() * g.element_size())
            work.wait()
        else:
            dist.reduce_scatter_tensor(out, g, group=ctx.group)
        return out


class _SPScatter(Function):
    """Partial sums [N n, H] -> this rank's [n, H] token shard of their sum over
    the forward group (reduce-scatter); backward: all-gather."""

    @staticmethod
    def forward(ctx, x: torch.Tensor) -> torch.Tensor:
        group = _fwd_group()
        W = _group_size(group)
        ctx.group = group
        x = x.contiguous()
        if x.shape[0] % W:
            raise ValueError(f"sequence parallelism: {x.shape[0]} tokens do not split over {W} ranks")
        out = torch.empty((x.shape[0] // W,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(out, x, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        W = _group_size(ctx.group)
        out = torch.empty((W * g.shape[0],) + tuple(g.shape[1:]), dtype=g.dtype, device=g.device)
        dist.all_gather_into_tensor(out, g, group=ctx.group)
        return out


def sp_gather(x: torch.Tensor) -> torch.Tensor:
    """All tokens [N n, H] from the token shards [n, H] (sequence parallelism)."""
    return _SPGather.apply(x)


def sp_scatter(x: torch.Tensor) -> torch.Tensor:
    """This rank's token shard of the sum over the ranks of x [N n, H]."""
    return _SPScatter.apply(x)


def mark_deferred_gategrads(model: nn.Module) -> int:
    """Let every gated layer inside a module whose input passes through the
    f operator (attention, MLP) defer its gate-gradient GEMM until that
    module's input-gradient all-reduce is in flight.  Returns the count."""
    n = 0
    for mod in model.modules():
        if not getattr(mod, "_tp_input_copy", False):
            continue
        for sub in mod.modules():
            if hasattr(sub, "gates") and hasattr(sub, "candidate_types") and sub is not mod:
                sub._defer_gategrad = True
                n += 1
    return n


def barrier() -> None:
    if TP.enabled and dist.is_initialized():
        dist.barrier()


def is_main_process() -> bool:
    return TP.rank == 0


class _AllReduceSum(Function):
    """All-reduce SUM forward, identity backward (reference parallel.py:140-160)."""

    @staticmethod
    def forward(ctx, t: torch.Tensor) -> torch.Tensor:
        out = t.clone().contiguous()
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=_fwd_group())
        return out

    @staticmethod
    def backward(ctx, g):
        return g


class _CopyToParallel(Function):
    """Identity forward, all-reduce SUM backward (exact dX at column-parallel inputs)."""

    @staticmethod
    def forward(ctx, t: torch.Tensor) -> torch.Tensor:
        return t.view_as(t)

    @staticmethod
    def backward(ctx, g):
        from voodoo_quant import layers

        if layers.has_deferred_gategrads():
            # the module's gate-gradient GEMMs run while the sum is in flight;
            # g is the sum of this module's gated layers' fresh input
            # gradients, so it is reduced in place
            g = g.contiguous()
            work = tp_all_reduce_async(g, overlap=True)
            layers.flush_deferred_gategrads(overlap_bytes=g.numel() * g.element_size())
            work.wait()
        else:
            g = g.clone().contiguous()
            dist.all_reduce(g, op=dist.ReduceOp.SUM, group=TP.group)
        return g


def tp_all_reduce_sum(t: torch.Tensor) -> torch.Tensor:
    if not TP.enabled:
        return t
    return _AllReduceSum.apply(t)


all_reduce_sum = tp_all_reduce_sum


class _AllReduceSumInPlace(Function):
    """`_AllReduceSum` without the copy: the input is summed in place."""

    @staticmethod
    def forward(ctx, t: torch.Tensor) -> torch.Tensor:
        ctx.mark_dirty(t)
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=_fwd_group())
        return t

    @staticmethod
    def backward(ctx, g):
        return g


def tp_all_reduce_sum_(t: torch.Tensor) -> torch.Tensor:
    """In-place `tp_all_reduce_sum` for a freshly produced contiguous tensor
    nothing else holds (a GEMM or lookup output): saves the copy of a
    [tokens, hidden] activation per row-parallel layer.  Autograd rejects it
    (version check) if the producer saved the tensor for its backward; a
    view that needs a gradient takes the copying path."""
    if not TP.enabled:
        return t
    if not t.is_contiguous():
        return tp_all_reduce_sum(t)
    if torch.is_grad_enabled() and t.requires_grad:
        if t._is_view():
            return tp_all_reduce_sum(t)
        return _AllReduceSumInPlace.apply(t)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=_fwd_group())
    return t


def all_reduce_(t: torch.Tensor) -> torch.Tensor:
    """Plain in-place SUM over the TP group, outside autograd (a no-op without TP)."""
    if TP.enabled:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=_fwd_group())
    return t


class _NcclRowReducer:
    """Row-parallel GEMM whose fresh output is summed over the TP ranks in
    place by NCCL (used inside the gated Linear's forward)."""

    @staticmethod
    def linear(x2: torch.Tensor, w: torch.Tensor, n_out: int, in_features: int) -> torch.Tensor:
        from voodoo_quant import _C

        y = _C.linear_fwd(x2, w, n_out, in_features)
        return all_reduce_(y)


_NCCL_ROW_REDUCER = _NcclRowReducer()


class _AsyncRowReducer:
    """`_NcclRowReducer` that only starts the in-place all-reduce (inside
    ``deferred_row_sums``); the handle goes to ``take_row_sums``."""

    @staticmethod
    def linear(x2: torch.Tensor, w: torch.Tensor, n_out: int, in_features: int) -> torch.Tensor:
        from voodoo_quant import _C

        y = _C.linear_fwd(x2, w, n_out, in_features)
        _ROW_SUMS.append(dist.all_reduce(y, op=dist.ReduceOp.SUM, group=_fwd_group(), async_op=True))
        return y


_ASYNC_ROW_REDUCER = _AsyncRowReducer()


def nccl_row_reducer():
    """The in-place NCCL reducer for row-parallel gated Linears (None without
    TP); inside ``deferred_row_sums`` the one that leaves the sum in flight."""
    if not TP.enabled:
        return None
    return _ASYNC_ROW_REDUCER if TP.defer_row_sums else _NCCL_ROW_REDUCER


def tp_copy_to_parallel(t: torch.Tensor) -> torch.Tensor:
    if not TP.enabled or not TP.exact_input_grad or TP.sequence_parallel:
        return t  # (under sequence parallelism the block's input all-gather sums it in backward)
    return _CopyToParallel.apply(t)


class _Done:
    def wait(self):
        return None


def tp_all_reduce_async(t: torch.Tensor, overlap: bool = False):
    """In-place all-reduce SUM of `t` on the TP group, returning a handle to
    wait on (a no-op handle when TP is disabled).  `overlap`: on the
    communicator of the collectives that run beside GEMMs, when there is one."""
    if not TP.enabled:
        return _Done()
    group = TP.overlap_group if overlap and TP.overlap_group is not None else TP.group
    return dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group, async_op=True)


def tp_broadcast(t: torch.Tensor, src: int = 0) -> torch.Tensor:
    if TP.enabled:
        dist.broadcast(t, src=src, group=TP.group)
    return t


def all_reduce_gate_grads(params) -> None:
    """Sum the gate gradients of every rank with ONE flat all-reduce.

    Same result as the reference's per-tensor loop (trainer.py:434-444); the
    order of tensors inside the flat buffer is the (identical) parameter order
    on every rank.
    """
    if not TP.enabled:
        return
    params = [p for p in params if p.grad is not None]
    if not params:
        return
    dt = params[0].grad.dtype
    for p in params[1:]:
        dt = torch.promote_types(dt, p.grad.dtype)
    flat = torch.cat([p.grad.reshape(-1).to(dt) for p in params])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=TP.group)
    off = 0
    for p in params:
        n = p.grad.numel()
        p.grad.copy_(flat[off:off + n].view_as(p.grad))
        off += n


def block_aligned_split(total: int, world: int, rank: int, unit: int = UNIT) -> tuple[int, int]:
    """(offset, length) of rank's share of `total`, in whole `unit`s, as even as possible.

    The first (units % world) ranks get one extra unit.  Raises ValueError when
    `total` is not a multiple of `unit` or some rank would get nothing.
    """
    if total % unit:
        raise ValueError(f"dimension {total} is not a multiple of the {unit}-element block")
    units = total // unit
    if units < world:
        raise ValueError(f"dimension {total} has {units} blocks, fewer than {world} ranks")
    base, extra = divmod(units, world)
    start = rank * base + min(rank, extra)
    n = base + (1 if rank < extra else 0)
    return start * unit, n * unit


def even_split(total: int, world: int, rank: int) -> tuple[int, int]:
    if total % world:
        raise ValueError(f"dimension {total} not divisible by tp={world}")
    n = total // world
    return rank * n, n


@dataclass
class ShardSpec:
    """Maps a rank-local slice back to its FULL tensor (reference parallel.py:183-299)."""

    full_out: int
    full_in: int
    row_offset: int | None = None
    row_len: int | None = None
    row_index: torch.Tensor | None = None
    col_offset: int | None = None
    col_len: int | None = None
    vocab_start: int | None = None
    # row-parallel slice whose ends need not fall on a 256-weight block: the
    # rank stores the blocks covering its columns (see in_col_offset)
    halo: bool = False

    def col_units(self) -> tuple[int, int]:
        """First and one-past-last 256-weight unit of the packed row that
        this rank stores (the units covering its columns)."""
        c0 = self.col_offset or 0
        c1 = c0 + self.local_in
        return c0 // UNIT, (c1 + UNIT - 1) // UNIT

    @property
    def in_col_offset(self) -> int:
        """Column of the rank's first input inside its stored blocks: 0
        unless a halo slice starts inside a block."""
        if not self.halo or self.col_offset is None:
            return 0
        return self.col_offset - self.col_units()[0] * UNIT

    @property
    def local_out(self) -> int:
        if self.row_index is not None:
            return int(self.row_index.numel())
        if self.row_len is not None:
            return self.row_len
        return self.full_out

    @property
    def local_in(self) -> int:
        return self.col_len if self.col_len is not None else self.full_in

    def describe(self) -> str:
        kind = "row-grouped" if self.row_index is not None else (
            "column" if self.row_len is not None else ("row" if self.col_len is not None else "none"))
        return f"{kind}-parallel local [{self.local_out}x{self.local_in}] of full [{self.full_out}x{self.full_in}]"

    def slice_weight(self, w_full: torch.Tensor) -> torch.Tensor:
        if self.row_index is not None:
            w = w_full[self.row_index.to(w_full.device)]
        elif self.row_offset is not None:
            w = w_full[self.row_offset:self.row_offset + self.row_len]
        else:
            w = w_full
        if self.col_offset is not None:
            w = w[:, self.col_offset:self.col_offset + self.col_len]
        return w

    def slice_qbytes(self, qb_full: torch.Tensor, quant_type: str, padded_full_in: int) -> torch.Tensor:
        """Slice FULL packed blocks to this rank's rows / block-aligned columns."""
        from voodoo_quant.ggml import get_quant_info

        info = get_quant_info(quant_type)
        bs, bb = info.block_size, info.block_bytes
        if padded_full_in % bs != 0:
            raise ValueError(f"{quant_type}: padded in {padded_full_in} not block-aligned ({bs})")
        nbpr = padded_full_in // bs
        if qb_full.numel() != self.full_out * nbpr * bb:
            raise ValueError(f"{quant_type}: qbytes numel {qb_full.numel()} != "
                             f"{self.full_out}x{nbpr}x{bb} expected for the FULL tensor")
        q2 = qb_full.reshape(self.full_out, nbpr, bb)
        if self.row_index is not None:
            q2 = q2[self.row_index.to(q2.device)]
        elif self.row_offset is not None:
            q2 = q2[self.row_offset:self.row_offset + self.row_len]
        if self.col_offset is not None:
            if self.halo:
                u0, u1 = self.col_units()
                q2 = q2[:, u0 * UNIT // bs:u1 * UNIT // bs]
                return q2.reshape(-1, bb)
            if self.col_offset % UNIT or self.col_len % UNIT:
                raise ValueError(
                    f"{quant_type}: column slice [{self.col_offset}:{self.col_offset + self.col_len}] is not "
                    f"aligned to the {UNIT}-weight block; TP shard boundaries must be block-aligned")
            q2 = q2[:, self.col_offset // bs:(self.col_offset + self.col_len) // bs]
        return q2.reshape(-1, bb)

    def local_padded_in(self, padded_full_in: int, candidate_types: list[str]) -> int:
        if self.col_len is None:
            return padded_full_in
        if self.halo:
            u0, u1 = self.col_units()
            return (u1 - u0) * UNIT
        if self.col_len % UNIT:
            raise ValueError(f"the rank-local input slice {self.col_len} is not a multiple of {UNIT}; "
                             "use block_aligned_split for row-parallel shards")
        return self.col_len

    def local_block_weight(self, w_full: torch.Tensor) -> torch.Tensor:
        """This rank's rows of the full tensor over the 256-weight units it
        stores (every unit without a column shard; the covering units of a
        halo shard), zero-padded past the full width.  The packed formats are
        block-local, so packing this gives exactly the blocks ``slice_qbytes``
        keeps of the packed full tensor, at 1/world of the packing work."""
        w = w_full
        if self.row_index is not None:
            w = w[self.row_index.to(w.device)]
        elif self.row_offset is not None:
            w = w[self.row_offset:self.row_offset + self.row_len]
        u0, u1 = self.col_units()
        w = w[:, u0 * UNIT:min(u1 * UNIT, w.shape[1])]
        if w.shape[1] < (u1 - u0) * UNIT:
            w = F.pad(w, (0, (u1 - u0) * UNIT - w.shape[1]))
        return w.contiguous()


class ColumnParallelLinear(nn.Linear):
    """Output rows sharded; no communication in forward."""

    def __init__(self, weight_slice: torch.Tensor, spec: ShardSpec, full_weight: torch.Tensor,
                 vocab_start: int | None = None):
        super().__init__(spec.full_in, spec.local_out, bias=False, device="meta", dtype=weight_slice.dtype)
        self.weight = nn.Parameter(weight_slice, requires_grad=False)
        self.tp_shard_spec = spec
        self.tp_full_weight = full_weight
        if vocab_start is not None:
            self.tp_vocab_start = vocab_start
            self.tp_vocab_end = vocab_start + spec.local_out


class RowParallelLinear(nn.Linear):
    """Input columns sharded; forward all-reduces the partial sums."""

    def __init__(self, weight_slice: torch.Tensor, spec: ShardSpec, full_weight: torch.Tensor):
        super().__init__(spec.local_in, spec.full_out, bias=False, device="meta", dtype=weight_slice.dtype)
        self.weight = nn.Parameter(weight_slice.contiguous(), requires_grad=False)
        self.tp_shard_spec = spec
        self.tp_full_weight = full_weight

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = F.linear(x.to(self.weight.device), self.weight)
        return y if sp_enabled() else tp_all_reduce_sum(y)


class VocabParallelEmbedding(nn.Embedding):
    """Vocabulary rows sharded; masked lookup + all-reduce."""

    def __init__(self, weight_slice: torch.Tensor, spec: ShardSpec, full_weight: torch.Tensor):
        super().__init__(spec.local_out, spec.full_in, device="meta", dtype=weight_slice.dtype)
        self.weight = nn.Parameter(weight_slice)
        self.tp_shard_spec = spec
        self.tp_full_weight = full_weight
        self.tp_vocab_start = spec.vocab_start
        self.tp_vocab_end = spec.vocab_start + spec.local_out

    def forward(self, input: torch.Tensor) -> torch.Tensor:
        input = input.to(self.weight.device)
        v0, v1 = self.tp_vocab_start, self.tp_vocab_end
        mask = (input < v0) | (input >= v1)
        out = F.embedding((input - v0).clamp(0, self.num_embeddings - 1), self.weight)
        out = out * (~mask).unsqueeze(-1).to(out.dtype)
        return out if sp_enabled() else tp_all_reduce_sum(out)


_PARALLEL_TYPES = (ColumnParallelLinear, RowParallelLinear, VocabParallelEmbedding)


def _shard_child(parent: nn.Module, name: str, *, row_offset=None, row_len=None, row_index=None,
                 col_offset=None, col_len=None, vocab_start=None, halo: bool = False) -> nn.Module:
    """Replace parent.<name> (nn.Linear / nn.Embedding) with its rank-local parallel module."""
    child = getattr(parent, name)
    if isinstance(child, _PARALLEL_TYPES):
        return child
    if isinstance(child, nn.Linear):
        w = child.weight.data
        spec = ShardSpec(full_out=w.shape[0], full_in=w.shape[1], row_offset=row_offset, row_len=row_len,
                         row_index=row_index, col_offset=col_offset, col_len=col_len, vocab_start=vocab_start,
                         halo=halo and col_offset is not None)
        sl = spec.slice_weight(w)
        new = ColumnParallelLinear(sl, spec, w, vocab_start) if col_offset is None else RowParallelLinear(sl, spec, w)
        setattr(parent, name, new)
        return new
    if isinstance(child, nn.Embedding):
        w = child.weight.data
        if vocab_start is None:
            raise ValueError("embedding sharding requires vocab_start")
        spec = ShardSpec(full_out=w.shape[0], full_in=w.shape[1], row_offset=row_offset, row_len=row_len,
                         vocab_start=vocab_start)
        new = VocabParallelEmbedding(spec.slice_weight(w), spec, w)
        setattr(parent, name, new)
        return new
    raise TypeError(f"parallel: cannot shard {type(child).__name__} at '{name}'")


def _install_input_copy(module: nn.Module) -> None:
    """Route the first positional / `hidden_states` input through the f operator."""
    if getattr(module, "_tp_input_copy", False):
        return

    def hook(mod, args, kwargs):
        if args:
            return (tp_copy_to_parallel(args[0]),) + tuple(args[1:]), kwargs
        if "hidden_states" in kwargs:
            kwargs = dict(kwargs)
            kwargs["hidden_states"] = tp_copy_to_parallel(kwargs["hidden_states"])
        return args, kwargs

    module.register_forward_pre_hook(hook, with_kwargs=True)
    module._tp_input_copy = True


def tp_mlp(mlp: nn.Module) -> None:
    """gate/up column-parallel, down row-parallel (uneven 256-aligned split allowed)."""
    tp, r = TP.world_size, TP.rank
    off, n = block_aligned_split(mlp.gate_proj.out_features, tp, r)
    _shard_child(mlp, "gate_proj", row_offset=off, row_len=n)
    _shard_child(mlp, "up_proj", row_offset=off, row_len=n)
    _shard_child(mlp, "down_proj", col_offset=off, col_len=n)
    _install_input_copy(mlp)


def tp_attention_dense(attn: nn.Module, num_heads: int, num_kv_heads: int, head_dim: int) -> None:
    """Llama-style attention: q/k/v column-parallel by whole heads, o row-parallel.

    o_proj's rank-local input is the rank's heads; when that width is not a
    multiple of the 256-weight block (40 heads x 128 at TP-8 = 640 columns)
    the o_proj shard is a halo shard (``ShardSpec.halo``), so heads and GQA
    groups stay whole.
    """
    tp, r = TP.world_size, TP.rank
    if num_heads % tp or num_kv_heads % tp:
        raise ValueError(f"attention heads ({num_heads} q / {num_kv_heads} kv) must divide tp={tp}")
    hq, hk = num_heads // tp, num_kv_heads // tp
    width = hq * head_dim
    if width % UNIT and width % 8:
        raise ValueError(f"o_proj rank-local input {width} is neither 256-block aligned nor a multiple of 8")
    _shard_child(attn, "q_proj", row_offset=r * hq * head_dim, row_len=hq * head_dim)
    _shard_child(attn, "k_proj", row_offset=r * hk * head_dim, row_len=hk * head_dim)
    _shard_child(attn, "v_proj", row_offset=r * hk * head_dim, row_len=hk * head_dim)
    _shard_child(attn, "o_proj", col_offset=r * width, col_len=width, halo=width % UNIT != 0)
    attn.tp_heads_local = hq
    _install_input_copy(attn)


def tp_attention(attn: nn.Module) -> None:
    """Gated attention whose q_proj emits a (q | gate) pair per head (the
    reference's Qwen3.5 adapter, parallel.py:563-591): q_proj, k_proj and
    v_proj split into contiguous equal row ranges -- whole heads, each head's
    q and gate together -- and o_proj by the matching input columns; the
    module's own forward then runs on the local heads."""
    tp, r = TP.world_size, TP.rank
    q, k, o = attn.q_proj, attn.k_proj, attn.o_proj
    head_dim = getattr(attn, "head_dim", 0) or 1
    if q.out_features % tp:
        raise ValueError(f"q_proj out {q.out_features} not divisible by tp={tp}")
    if k.out_features % (tp * head_dim):
        raise ValueError(f"k_proj out {k.out_features} does not split into whole heads over tp={tp} "
                         f"(head_dim {head_dim}); the TP degree must divide the KV-head count")
    nq = q.out_features // tp
    _shard_child(attn, "q_proj", row_offset=r * nq, row_len=nq)
    for name in ("k_proj", "v_proj"):
        m = getattr(attn, name)
        if m.out_features % tp:
            raise ValueError(f"{name} out {m.out_features} not divisible by tp={tp}")
        n = m.out_features // tp
        _shard_child(attn, name, row_offset=r * n, row_len=n)
    if o.in_features % tp:
        raise ValueError(f"o_proj in {o.in_features} not divisible by tp={tp}")
    no = o.in_features // tp
    _shard_child(attn, "o_proj", col_offset=r * no, col_len=no)
    attn.tp_heads_local = q.out_features // (2 * head_dim * tp)
    _install_input_copy(attn)


def tp_ssm(gdn: nn.Module) -> None:
    """Gated DeltaNet block sharded by value heads, key heads in lockstep (the
    reference's Qwen3.5 adapter, parallel.py:594-646).

    in_proj_qkv emits [q (key_dim) | k (key_dim) | v (value_dim)]; the rank
    keeps its slice of each of the three, concatenated in that order, which is
    also the channel order of the depthwise conv and of the module's split,
    so the conv, the per-head dt_bias / A_log and the dimension attributes are
    made rank-local the same way and the stock forward runs unchanged.
    in_proj_z / in_proj_b / in_proj_a split by rows, out_proj by columns.
    """
    tp, r = TP.world_size, TP.rank
    kd, vd, nv = gdn.key_dim, gdn.value_dim, gdn.num_v_heads
    if kd % tp or vd % tp or nv % tp or gdn.num_k_heads % tp:
        raise ValueError(f"SSM dims (key {kd}, value {vd}, v-heads {nv}, k-heads {gdn.num_k_heads}) "
                         f"not divisible by tp={tp}")
    kl, vl, nvl = kd // tp, vd // tp, nv // tp
    keep = torch.cat([torch.arange(r * kl, (r + 1) * kl), torch.arange(kd + r * kl, kd + (r + 1) * kl),
                      torch.arange(2 * kd + r * vl, 2 * kd + (r + 1) * vl)])
    _shard_child(gdn, "in_proj_qkv", row_index=keep)
    _shard_child(gdn, "in_proj_z", row_offset=r * vl, row_len=vl)
    _shard_child(gdn, "in_proj_b", row_offset=r * nvl, row_len=nvl)
    _shard_child(gdn, "in_proj_a", row_offset=r * nvl, row_len=nvl)
    _shard_child(gdn, "out_proj", col_offset=r * vl, col_len=vl)
    conv = gdn.conv1d
    channels = 2 * kl + vl
    pad = conv.padding[0] if isinstance(conv.padding, tuple) else conv.padding
    local = nn.Conv1d(channels, channels, kernel_size=conv.kernel_size, groups=channels, padding=pad,
                      bias=conv.bias is not None)
    with torch.no_grad():
        local.weight.copy_(conv.weight.data[keep.to(conv.weight.device)])
        if conv.bias is not None:
            local.bias.copy_(conv.bias.data[keep.to(conv.bias.device)])
    gdn.conv1d = local.to(conv.weight.device, conv.weight.dtype)
    with torch.no_grad():
        gdn.dt_bias.data = gdn.dt_bias.data[r * nvl:(r + 1) * nvl].clone()
        gdn.A_log.data = gdn.A_log.data[r * nvl:(r + 1) * nvl].clone()
    gdn.num_v_heads, gdn.num_k_heads = nvl, gdn.num_k_heads // tp
    gdn.key_dim, gdn.value_dim, gdn.conv_dim = kl, vl, channels
    _install_input_copy(gdn)


def _slice_q8_bytes(qb: torch.Tensor, full_out: int, full_in: int, row_index=None, row_range=None,
                    col_range=None) -> torch.Tensor:
    """Rank-local Q8_0 bytes ([nblocks, 34], 32 weights per block) of a full
    tensor's blocks, by row index, row range and/or 32-aligned column range
    (reference parallel.py:393-408)."""
    q = qb.reshape(full_out, full_in // 32, 34)
    if row_index is not None:
        q = q[row_index.to(q.device)]
    elif row_range is not None:
        q = q[row_range[0]:row_range[1]]
    if col_range is not None:
        c0, c1 = col_range
        if c0 % 32 or (c1 - c0) % 32:
            raise ValueError(f"Q8_0 column slice [{c0}:{c1}] not 32-aligned")
        q = q[:, c0 // 32:c1 // 32]
    return q.reshape(-1, 34).contiguous()


def _shard_lm_head(model: nn.Module) -> None:
    head, holder = None, None
    for h, attr in ((model, "lm_head"), (getattr(model, "model", None), "lm_head")):
        if h is not None and getattr(h, attr, None) is not None:
            head, holder = getattr(h, attr), h
            break
    if head is None or isinstance(head, ColumnParallelLinear):
        return
    off, n = even_split(head.out_features, TP.world_size, TP.rank)
    new = _shard_child(holder, "lm_head", row_offset=off, row_len=n, vocab_start=off)
    # the final hidden state feeds only this vocab shard on each rank: its
    # gradient is the sum over the ranks' shards (f operator on the head input)
    _install_input_copy(new)


def tp_patch_model(model: nn.Module, verbose: bool = True) -> nn.Module:
    """Shard a model in place for the current rank via its registered arch adapter."""
    from voodoo_quant.arch import adapter_for_model

    adapter = adapter_for_model(model)
    if adapter is None:
        raise RuntimeError(
            f"no architecture adapter registered for {type(model).__name__} "
            f"(model_type={getattr(getattr(model, 'config', None), 'model_type', '?')}); "
            "tensor parallelism is refused rather than sharded blindly.")
    text = getattr(model, "model", None)
    if text is None or not hasattr(text, "layers"):
        text = model
    embed = getattr(text, "embed_tokens", None)
    if embed is not None:
        off, n = even_split(embed.num_embeddings, TP.world_size, TP.rank)
        _shard_child(text, "embed_tokens", row_offset=off, row_len=n, vocab_start=off)
    handled = 0
    for layer in text.layers:
        handled += len(adapter.shard_layer(layer))
    _shard_lm_head(model)
    if verbose and TP.rank == 0:
        print(f"[tp] patched rank {TP.rank}/{TP.world_size} ({adapter.__name__}): {handled} submodule groups",
              flush=True)
    return model
