"""The gated-candidate distillation step (the hot loop of training/trainer.py).

Keeps the reference step's semantics (voodoo_quant/training/trainer.py:
2443-2666) and helper names:

* temperature  tau_s = start * (end / start) ** (s / (S - 1))        (:199-203)
* loss         CE + distill_weight * T^2 * KL(teacher || student)    (:2567-2575)
               on the fused B200 loss kernel (``training.loss``)
* size         bytes = sum of effective_bytes + non-targeted 8-bit bytes;
               size_loss = relu(|bytes / target - 1| - tolerance)^2  (:2577-2590)
* optimiser    AdamW(gates, lr, betas=(0.9, 0.95)), clip-norm 1.0, cosine LR
               with eta_min 1e-3 (:2378-2379, :2607-2616); under TP the gate
               gradients are summed with one flat all-reduce first.

Only the gates train; every other parameter is frozen, as in the reference
(:2344-2351).
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass

import torch
import torch.nn as nn

from voodoo_quant.layers import GateBank, set_ptqr, set_static_shapes
from voodoo_quant.training.loss import chunked_head_loss, distillation_loss, tp_distillation_loss


def anneal_temperature(step: int, max_steps: int, start: float, end: float) -> float:
    if max_steps <= 1:
        return end
    frac = step / (max_steps - 1)
    return start * (end / start) ** frac


def compute_total_8bit_bytes(state_dict_meta: dict[str, tuple[int, int]]) -> float:
    """Bytes at 8 bits per parameter, shared storages counted once (:157-178)."""
    seen, total = set(), 0.0
    for ptr, numel in state_dict_meta.values():
        if ptr not in seen:
            seen.add(ptr)
            total += float(numel)
    return total


def compute_non_targeted_8bit_bytes(state_dict_meta: dict[str, tuple[int, int]], targeted_keys: set[str]) -> float:
    """8-bit bytes of parameters that are not gated (:181-196)."""
    ptr_bytes, ptr_targeted = {}, {}
    for k, (ptr, numel) in state_dict_meta.items():
        ptr_bytes[ptr] = float(numel)
        ptr_targeted.setdefault(ptr, False)
        if k in targeted_keys:
            ptr_targeted[ptr] = True
    return sum(b for p, b in ptr_bytes.items() if not ptr_targeted[p])


def state_dict_meta(model: nn.Module) -> dict[str, tuple[int, int]]:
    return {n: (t.untyped_storage().data_ptr(), t.numel()) for n, t in model.state_dict(keep_vars=True).items()
            if t.is_floating_point()}


def _tp_all_reduce_gate_grads(trainable) -> None:
    from voodoo_quant.parallel import all_reduce_gate_grads

    all_reduce_gate_grads(trainable)


@dataclass
class StepArgs:
    lr: float = 0.5
    distill_weight: float = 1.0
    distill_temperature: float = 1.0
    size_weight: float = 10.0
    size_tolerance: float = 0.02
    temp_start: float = 1.0
    temp_end: float = 0.01
    max_steps: int = 50
    ce_reduction: str = "valid"  # plain path: mean CE over non-ignored tokens
    ptqr: bool = False  # per-token quant routing forward (reference --ptqr, trainer.py:1523,1612-1616)
    # head + loss per chunk of this many tokens, never materialising the
    # [tokens, V] logits (reference --logits_chunk, trainer.py:753-832); 0 = off
    logits_chunk: int = 0
    # no host round trip in forward_backward (layers.set_static_shapes), so it
    # can be recorded as a CUDA graph (GatedDistillTrainer.capture); needs
    # ce_reduction="tokens" (the "valid" count is read on the host), which
    # equals "valid" whenever no target is ignored
    static_shapes: bool = False
    # TP degree of the teacher (0 = the student's): the teacher is sharded t
    # ways inside groups of t consecutive ranks, each group runs it on its
    # slice of the batch (the batch divides into world / t slices), and one
    # all-to-all hands every rank its vocabulary slice of all the teacher's
    # logits; each teacher all-reduce then moves 1 / (world / t) of the
    # tokens among t ranks.  Plain loss path only (logits_chunk = 0).
    teacher_tp: int = 0
    # under TP: sequence parallelism (parallel.enable_sequence_parallel) --
    # the residual stream, RMSNorms and residual adds on token shards, an
    # all-gather before and a reduce-scatter after every block instead of
    # the all-reduces of replicated activations
    sequence_parallel: bool = False
    # under TP with a teacher at TP-1 on its batch slice (teacher_tp = 1):
    # run the teacher's layers interleaved with the student's, each teacher
    # block issued while the student block's forward all-reduce is in flight
    # (its GEMMs leaving `joint_teacher_sms` SMs to the all-reduce)
    joint_teacher: bool = False
    joint_teacher_sms: int = 32


class GatedDistillTrainer:
    """Runs gated-candidate distillation steps on a replaced student model."""

    def __init__(self, student: nn.Module, teacher: nn.Module, replaced: dict, args: StepArgs,
                 target_bytes: float, non_targeted_bytes: float, tp: bool = False):
        self.student, self.teacher, self.replaced, self.args = student, teacher, replaced, args
        self.target_bytes = float(target_bytes)
        self.non_targeted_bytes = float(non_targeted_bytes)
        self.tp = tp
        for p in student.parameters():
            p.requires_grad = False
        for layer in replaced.values():
            layer.gates.requires_grad = True
        self.trainable = [layer.gates for layer in replaced.values()]
        self.bank = GateBank(replaced)  # every layer's softmax(g / tau) in one batched op per step
        set_ptqr(args.ptqr)
        if args.static_shapes and args.ce_reduction != "tokens" and args.logits_chunk <= 0:
            raise ValueError("static_shapes needs ce_reduction='tokens': the 'valid' token count is read on the host")
        set_static_shapes(args.static_shapes)
        self._graph = None
        self._tsplit = None  # (group, group index, rank in group, t) with a teacher of its own TP degree
        self.optimizer = torch.optim.AdamW(self.trainable, lr=args.lr, betas=(0.9, 0.95))
        self.scheduler = torch.optim.lr_scheduler.CosineAnnealingLR(self.optimizer, T_max=args.max_steps,
                                                                    eta_min=1e-3)
        self.step_idx = 0
        student.train()
        teacher.eval()

    def _vocab_start(self) -> int | None:
        head = getattr(self.student, "lm_head", None)
        return getattr(head, "tp_vocab_start", None)

    def forward_backward(self, x: torch.Tensor, y: torch.Tensor) -> dict:
        """Loss of one batch and its gate gradients (left in ``gates.grad``)."""
        a = self.args
        tau = anneal_temperature(self.step_idx, a.max_steps, a.temp_start, a.temp_end)
        if a.static_shapes:
            if not _capturing():  # a recorded step reads the scalar; replay_step sets it
                self.bank.set_temperature(tau)
        else:
            for layer in self.replaced.values():
                layer.set_temperature(tau)
        self.optimizer.zero_grad(set_to_none=True)
        self.bank.probs()
        v0 = self._vocab_start()
        if a.logits_chunk > 0:
            return self._forward_backward_chunked(x, y, a, tau, v0)
        if self._joint_ok():
            logits, t_logits = self._joint_forward(x)
        else:
            logits = self.student(input_ids=x, use_cache=False).logits
            with torch.no_grad():
                t_logits = self._teacher_logits(x)
        if self.tp and v0 is not None:
            kd, lm, kl = tp_distillation_loss(logits, t_logits, y, v0, a.distill_temperature, a.distill_weight,
                                              ce_reduction="tokens", unit_upstream=True)
        else:
            kd, lm, kl = distillation_loss(logits, t_logits, y, a.distill_temperature, a.distill_weight,
                                           ce_reduction=a.ce_reduction, unit_upstream=True)
        del t_logits
        current = self.bank.effective_bytes().to(logits.device)
        if self.tp:
            from voodoo_quant.parallel import tp_all_reduce_sum

            current = tp_all_reduce_sum(current)
        current = current + self.non_targeted_bytes
        rel = torch.abs(current / self.target_bytes - 1.0)
        size_loss = torch.relu(rel - a.size_tolerance) ** 2
        loss = kd + a.size_weight * size_loss
        loss.backward()
        self.bank.release()
        if self.tp:
            _tp_all_reduce_gate_grads(self.trainable)
        return {"loss": loss.detach(), "lm_loss": lm, "distill_loss": kl, "size_bytes": current.detach(),
                "size_loss": size_loss.detach(), "tau": tau}

    def _size_loss(self, device):
        a = self.args
        current = self.bank.effective_bytes().to(device)
        if self.tp:
            from voodoo_quant.parallel import tp_all_reduce_sum

            current = tp_all_reduce_sum(current)
        current = current + self.non_targeted_bytes
        rel = torch.abs(current / self.target_bytes - 1.0)
        return current, torch.relu(rel - a.size_tolerance) ** 2

    def _forward_backward_chunked(self, x, y, a: StepArgs, tau: float, v0) -> dict:
        """Stacks once, then head + loss per chunk of ``a.logits_chunk`` tokens
        (``loss.chunked_head_loss``), then one backward through the student
        stack and the gate bank.  While the chunks run, a gated head reads its
        probabilities from a detached leaf, so each chunk's backward stays in
        the head; the leaf's accumulated gradient joins the final backward."""
        student, teacher = self.student, self.teacher
        hidden = student.model(input_ids=x, use_cache=False).last_hidden_state
        with torch.no_grad():
            t_hidden = teacher.model(input_ids=x, use_cache=False).last_hidden_state
        head = student.lm_head
        row = head.__dict__.get("_bank_probs")
        bank_ref = head.__dict__.get("_bank_ref")
        leaf = row.detach().requires_grad_(True) if row is not None else None
        if leaf is not None:  # (PTQR: the head then draws its own routing per chunk)
            head._bank_probs, head._bank_ref = leaf, None
        try:
            h_grad, kd, lm, kl = chunked_head_loss(head, teacher.lm_head, hidden, t_hidden, y, a.logits_chunk,
                                                   a.distill_temperature, a.distill_weight,
                                                   vocab_start=v0 if self.tp else None)
        finally:
            if leaf is not None:
                head._bank_probs, head._bank_ref = row, bank_ref
        del t_hidden
        current, size_loss = self._size_loss(hidden.device)
        outs, grads = [hidden, a.size_weight * size_loss], [h_grad, None]
        if leaf is not None and leaf.grad is not None:
            outs.append(row)
            grads.append(leaf.grad)
        torch.autograd.backward(outs, grads)
        self.bank.release()
        if self.tp:
            _tp_all_reduce_gate_grads(self.trainable)
        loss = kd + a.size_weight * size_loss.detach()
        return {"loss": loss, "lm_loss": lm, "distill_loss": kl, "size_bytes": current.detach(),
                "size_loss": size_loss.detach(), "tau": tau}

    def _joint_ok(self) -> bool:
        """Whether this step interleaves the teacher with the student
        (StepArgs.joint_teacher; TP with a TP-1 teacher on the rank's batch
        slice, the plain loss path, no sequence parallelism)."""
        from voodoo_quant.parallel import sp_enabled

        a = self.args
        return (a.joint_teacher and self.tp and self._tsplit is not None and self._tsplit[3] == 1
                and a.logits_chunk <= 0 and not sp_enabled()
                and hasattr(getattr(self.student, "model", None), "layers")
                and hasattr(getattr(self.teacher, "model", None), "layers"))

    def _joint_forward(self, x: torch.Tensor):
        """Student logits (autograd) and teacher logits (no grad, in the
        student's vocabulary layout) with the teacher's decoder layers
        interleaved between the student's: each student block's row-parallel
        output is summed by an all-reduce started in place,
        the teacher's matching block is issued while it is in flight, and the
        student waits for the sum only when it reads it (row-parallel gated
        layers start their in-place sums inside ``deferred_row_sums``).  The
        same operations
        and sums as the two forwards one after the other."""
        from voodoo_quant import _C
        from voodoo_quant.parallel import TP, _fwd_group, deferred_row_sums, redistribute_vocab_shards, take_row_sums

        _, g, _, t = self._tsplit
        G = TP.world_size // t
        if x.shape[0] % G:
            raise ValueError(f"batch {x.shape[0]} does not split over {G} teacher groups (teacher_tp={t})")
        b = x.shape[0] // G
        xt = x[g * b:(g + 1) * b]
        sm, tm = self.student.model, self.teacher.model
        s_layers = sm.layers[: sm.config.num_hidden_layers]
        t_layers = tm.layers[: tm.config.num_hidden_layers]
        if len(s_layers) != len(t_layers):
            raise ValueError("joint teacher schedule needs as many teacher layers as student layers")
        hs = sm.embed_tokens(x)
        pe_s = sm.rotary_emb(hs, position_ids=torch.arange(hs.shape[1], device=hs.device).unsqueeze(0))
        with torch.no_grad():
            ht = tm.embed_tokens(xt)
            pe_t = tm.rotary_emb(ht, position_ids=torch.arange(ht.shape[1], device=ht.device).unsqueeze(0))

        @contextlib.contextmanager
        def beside_sum():  # the teacher's GEMMs leave SMs to the all-reduce in flight
            n = self.args.joint_teacher_sms
            if n > 0:
                _C.set_gemm_sm_reserve(n)
            try:
                with torch.no_grad():
                    yield
            finally:
                if n > 0:
                    _C.set_gemm_sm_reserve(0)

        pend_s = pend_t = None
        xt_n = None
        for ls, lt in zip(s_layers, t_layers):
            hs, xs = _res_norm(pend_s, hs, ls.input_layernorm)
            with deferred_row_sums():
                a = ls.self_attn(hidden_states=xs, attention_mask=None, position_embeddings=pe_s)[0]
            works = take_row_sums()  # o_proj's sum, in flight
            with beside_sum():
                ht, xt_n = _res_norm(pend_t, ht, lt.input_layernorm)
                at = lt.self_attn(hidden_states=xt_n, attention_mask=None, position_embeddings=pe_t)[0]
                ht, xt_n = _res_norm(at, ht, lt.post_attention_layernorm)
            for w in works:
                w.wait()
            hs, xs = _res_norm(a, hs, ls.post_attention_layernorm)
            with deferred_row_sums():
                m = ls.mlp(xs)
            works = take_row_sums()  # down_proj's sum, in flight
            with beside_sum():
                pend_t = lt.mlp(xt_n)
            for w in works:
                w.wait()
            pend_s = m
        hs, out_s = _res_norm(pend_s, hs, sm.norm)
        with torch.no_grad():
            _, out_t = _res_norm(pend_t, ht, tm.norm)
            t_local = self.teacher.lm_head(out_t)
        logits = self.student.lm_head(out_s)
        return logits, redistribute_vocab_shards(t_local, t, group=_fwd_group())

    def _teacher_logits(self, x: torch.Tensor) -> torch.Tensor:
        """The teacher's logits in the student's layout.  With a teacher of
        its own TP degree, this rank's group runs the teacher on its batch
        slice (collectives inside the group) and one all-to-all, on the
        communicator the forward's collectives use here, redistributes the
        vocabulary shards."""
        if self._tsplit is None:
            return self.teacher(input_ids=x, use_cache=False).logits
        from voodoo_quant.parallel import TP, _fwd_group, collectives_on, redistribute_vocab_shards

        group, g, _, t = self._tsplit
        G = TP.world_size // t
        if x.shape[0] % G:
            raise ValueError(f"batch {x.shape[0]} does not split over {G} teacher groups (teacher_tp={t})")
        b = x.shape[0] // G
        with collectives_on(group):
            local = self.teacher(input_ids=x[g * b:(g + 1) * b], use_cache=False).logits
        return redistribute_vocab_shards(local, t, group=_fwd_group())

    def apply_update(self) -> None:
        torch.nn.utils.clip_grad_norm_(self.trainable, max_norm=1.0)
        self.optimizer.step()
        self.scheduler.step()
        self.step_idx += 1

    def step(self, x: torch.Tensor, y: torch.Tensor) -> dict:
        out = self.forward_backward(x, y)
        self.apply_update()
        return out

    # ---- one CUDA graph per step (static_shapes) ----
    def capture(self, x: torch.Tensor, y: torch.Tensor, warmup: int = 3) -> None:
        """Record ``forward_backward`` on static copies of ``x`` / ``y`` as one
        CUDA graph: every kernel and collective of the forward and backward,
        launched by one replay instead of thousands of host calls.  The
        optimizer stays eager (clip, AdamW and the schedule are a few launches
        over the gates).  ``warmup`` eager steps run first on a side stream
        (workspaces, communicators, cuDNN plans); they use the gates as they
        are and update nothing."""
        if not self.args.static_shapes:
            raise RuntimeError("capture needs StepArgs(static_shapes=True)")
        self._gx, self._gy = x.clone(), y.clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.forward_backward(self._gx, self._gy)
        torch.cuda.current_stream().wait_stream(side)
        self.optimizer.zero_grad(set_to_none=True)
        torch.cuda.synchronize()
        torch.cuda.empty_cache()  # the graph allocates from its own pool: hand the warm-up's cache back
        self.bank.set_temperature(anneal_temperature(self.step_idx, self.args.max_steps, self.args.temp_start,
                                                     self.args.temp_end))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._gout = self.forward_backward(self._gx, self._gy)
        self._graph = graph

    def replay_step(self, x: torch.Tensor, y: torch.Tensor) -> dict:
        """One step through the recorded graph: this step's temperature into
        the bank's scalar, the batch into the static inputs, replay (the
        gates' gradients are rewritten in place), then the eager update.
        Returns the step's outputs (tensors owned by the graph, overwritten
        by the next replay)."""
        if self._graph is None:
            raise RuntimeError("replay_step needs capture() first")
        a = self.args
        tau = anneal_temperature(self.step_idx, a.max_steps, a.temp_start, a.temp_end)
        self.bank.set_temperature(tau)
        self._gx.copy_(x, non_blocking=True)
        self._gy.copy_(y, non_blocking=True)
        self._graph.replay()
        self.apply_update()
        out = dict(self._gout)
        out["tau"] = tau
        return out

    def release_graph(self) -> None:
        """Drop the recorded graph (before destroying a process group whose
        collectives it holds)."""
        self._graph = None
        self._gout = None

    def assignments(self) -> dict[str, str]:
        return {name: layer.get_assignment() for name, layer in self.replaced.items()}


def _res_norm(pending, h: torch.Tensor, norm):
    """(h + pending, norm(h + pending)), or (h, norm(h)) without a pending
    output: one add + RMSNorm kernel where the fused kernels apply."""
    if pending is None:
        return h, norm(h)
    from voodoo_quant.fused_blocks import _fusable, _norm_weights_fusable, add_rms_norm

    if _fusable(h) and _norm_weights_fusable(norm):
        return add_rms_norm(pending, h, norm.weight, norm.variance_epsilon)
    h = h + pending
    return h, norm(h)


def _capturing() -> bool:
    return torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()


def build_distill(shape_name: str, device, seed: int = 0, args: StepArgs | None = None,
                  candidate_provider=None, replace_embeddings: bool = True, tp: bool = False,
                  fused_blocks: bool = True, overlap_sms: int = 0):
    """Student (gated), Q8_0 teacher and trainer for a synthetic config.

    Under TP (an initialised process group adopted by voodoo_quant.parallel)
    both models are sharded by the Llama adapter before replacement, so the
    candidates are packed from the FULL tensors and sliced per rank.  On a
    CUDA device ``fused_blocks`` routes the Llama blocks' RMSNorm, rotary
    embedding and SwiGLU through the fused kernels (``voodoo_quant.fused_blocks``).
    Under TP with
    ``overlap_sms`` > 0, each attention / MLP block's gate-gradient GEMMs
    run beside the all-reduce of the block's input gradient on a second
    communicator limited to that many CTAs (``parallel.enable_input_grad_overlap``,
    ``parallel.mark_deferred_gategrads``); the GEMMs leave those SMs free.

    Shapes with per-role menus pass them on as the reference's
    ``--attention_candidates`` / ``--non_attention_candidates``.  The teacher
    is built after the student's full weights are released (both models draw
    the same seeded weights), so at most one full bf16 model is on the device
    at a time -- 61.5 GB for the 32B shape.
    """
    from voodoo_quant.layers import replace_embedding_with_mixed_quant, replace_linear_with_mixed_quant
    from voodoo_quant.parallel import TP, tp_patch_model
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.q8_teacher import wrap_q8_teacher

    shape = S.SHAPES[shape_name]
    provider = candidate_provider or S.rtn_candidate_provider
    menus = dict(attention_candidates=shape.attention_candidates,
                 non_attention_candidates=shape.non_attention_candidates)
    base = S.build_llama(shape, device, seed=seed)
    meta = state_dict_meta(base)
    total_8bit = compute_total_8bit_bytes(meta)
    if tp and TP.enabled:
        tp_patch_model(base, verbose=False)
    skip = {"lm_head"} if shape.tied else set()
    replaced = replace_linear_with_mixed_quant(base, shape.candidates, skip_names=skip, device=device,
                                               candidate_provider=provider, **menus)
    if replace_embeddings:
        replaced.update(replace_embedding_with_mixed_quant(base, shape.candidates, device=device,
                                                           candidate_provider=provider, **menus))
    targeted = {n + ".weight" for n in replaced}
    non_targeted = compute_non_targeted_8bit_bytes(meta, targeted)
    for m in base.modules():  # drop the full-weight references kept for candidate packing
        if hasattr(m, "tp_full_weight"):
            m.tp_full_weight = None
    if torch.device(device).type == "cuda":
        torch.cuda.empty_cache()
    teacher = S.build_llama(shape, device, seed=seed)
    tsplit = None
    if tp and TP.enabled:
        t = (args.teacher_tp if args is not None else 0) or TP.world_size
        if t != TP.world_size:
            from voodoo_quant.parallel import as_tp, teacher_subgroups

            if args.logits_chunk > 0:
                raise ValueError("teacher_tp needs the plain loss path (logits_chunk=0)")
            group, g, h = teacher_subgroups(t)
            if t > 1:
                with as_tp(h, t, group):
                    tp_patch_model(teacher, verbose=False)
            tsplit = (group, g, h, t)
        else:
            tp_patch_model(teacher, verbose=False)
    wrap_q8_teacher(teacher, S.q8_quantizer)
    if fused_blocks and torch.device(device).type == "cuda":
        from voodoo_quant.fused_blocks import fuse_llama_blocks

        fuse_llama_blocks(base, causal_batches=True)
        fuse_llama_blocks(teacher, causal_batches=True)
    if tp and TP.enabled:
        from voodoo_quant.parallel import enable_sequence_parallel

        sp = args is not None and args.sequence_parallel
        if sp:
            from voodoo_quant.fused_blocks import use_sequence_parallel

            use_sequence_parallel(base)
            use_sequence_parallel(teacher)
        enable_sequence_parallel(sp)
    if tp and TP.enabled:
        if overlap_sms > 0:
            from voodoo_quant.parallel import enable_input_grad_overlap, mark_deferred_gategrads

            if enable_input_grad_overlap(overlap_sms):
                mark_deferred_gategrads(base)
    torch.cuda.empty_cache()
    trainer = GatedDistillTrainer(base, teacher, replaced, args or StepArgs(), shape.budget * total_8bit,
                                  non_targeted, tp=tp and TP.enabled)
    trainer._tsplit = tsplit
    return trainer, shape
