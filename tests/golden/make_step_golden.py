"""Golden values of one whole distillation step, from the reference's own modules.

Run once, in a container that has the reference checkout (never by the tests
or on the GPU box):

    python tests/golden/make_step_golden.py --reference <path to voodoo-dyn-quant>

Workload: the CPU-runnable tiny step (2 layers, hidden 256, 4 heads, SwiGLU
768, vocabulary 4096, untied; K = 4 candidates Q4_K, Q5_K, Q6_K, Q8_0 on
every Linear and the embedding; Q8_0 teacher; batch 2 x 128 tokens; budget
45 % of the 8-bit bytes).

Inputs are made exactly as this build's step makes them, so a test can
rebuild them from the seeds: the weights by ``training/synthetic.py``'s
``build_llama`` (seeded N(0, 0.02), bf16), the packed candidates by the
round-to-nearest packer ``quants/rtn.py``, the teacher's Q8_0 bytes by
gguf-py 0.19.0 (which this build's Q8_0 rule matches byte for byte).  Both
files are loaded by path under other module names, because the reference's
package of the same name is the one imported here.

Reference side, in float32 on the host:
* student: ``replace_linear_with_mixed_quant`` / ``replace_embedding_with_mixed_quant``
  (voodoo_quant/layers.py:1908-2153) in dequant mode; each candidate is
  decoded by the reference's torch decoders (layers.py:62-213) and handed over
  through the reference's own candidate-cache file (``_combined_cache_path``,
  ``_tensor_hash``), which its ``_MixedQuantBase.__init__`` loads
  (layers.py:1112-1140); its gates get the recorded initial values;
* teacher: ``training/q8_teacher.wrap_q8_teacher`` on the Q8_0 bytes;
* step: ``anneal_temperature``, the plain-path loss of
  training/trainer.py:2538-2575 (inline in the reference's training loop, so
  restated here line for line), ``total_effective_bytes`` with
  ``compute_total_8bit_bytes`` / ``compute_non_targeted_8bit_bytes``, the
  relu-squared size term (:2577-2590), backward, ``clip_grad_norm_(1.0)``,
  AdamW(betas 0.9, 0.95) and the cosine schedule (:2378-2379, :2606-2616).

Two variants: ``default`` (the reference's argument defaults: CE + 1.0 KL at
T = 1, size weight 10, tolerance 0.02, lr 0.5, step 0 so tau = 1) and ``kd``
(T = 2, KL weight 0.7, size weight 0, step 7 of 50 so tau = 0.01^(7/49)),
which leaves only the kernel-dependent distillation gradient in the gates.

Writes ``step_golden.npz``: tokens, initial gates per tensor, and per variant
the loss terms, four rows of student logits, the gate gradients per tensor
(before clipping), the gates after the optimizer step and the assignments.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PKG = HERE.parent.parent / "voodoo-dyn-quant_b200" / "voodoo_quant"

SEED = 3
TOKEN_SEED = 5
GATE_SEED = 20261202
TYPES = ["Q4_K", "Q5_K", "Q6_K", "Q8_0"]
VARIANTS = {  # distill_temperature, distill_weight, size_weight, step index
    "default": (1.0, 1.0, 10.0, 0),
    "kd": (2.0, 0.7, 0.0, 7),
}
MAX_STEPS, LR, TEMP_START, TEMP_END, TOL, BUDGET = 50, 0.5, 1.0, 0.01, 0.02, 0.45
LOGIT_ROWS = 4


def _load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod  # dataclasses look their module up while it executes
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()

    scratch = Path(tempfile.mkdtemp(prefix="vq_step_golden_"))
    os.environ["TRITON_CACHE_DIR"] = str(scratch / "triton")
    os.environ["TORCHINDUCTOR_CACHE_DIR"] = str(scratch / "inductor")
    sys.path.insert(0, args.reference)

    import torch
    import torch.nn.functional as F
    from gguf import GGMLQuantizationType, quants as gq

    syn = _load("b200_synthetic", PKG / "training" / "synthetic.py")
    rtn = _load("b200_rtn", PKG / "quants" / "rtn.py")

    from voodoo_quant import layers as L
    from voodoo_quant.training import q8_teacher as Q8
    from voodoo_quant.training import trainer as TR

    torch.set_num_threads(max(os.cpu_count() or 1, 1))
    L._CANDIDATE_CACHE_ROOT = scratch / "candidates"  # the reference tree stays untouched
    decoders = {"Q8_0": L._dequantize_q8_0_gpu, "Q4_K": L._dequantize_q4_K_gpu,
                "Q5_K": L._dequantize_q5_K_gpu, "Q6_K": L._dequantize_q6_K_gpu}

    shape = syn.SHAPES["tiny"]
    assert shape.candidates == TYPES and not shape.tied

    def fp32_model():
        return syn.build_llama(shape, "cpu", seed=SEED).float()

    # ---- candidates through the reference's own cache files -------------------
    student = fp32_model()
    for name, mod in student.named_modules():
        if isinstance(mod, (torch.nn.Linear, torch.nn.Embedding)):
            w = mod.weight.detach().contiguous()
            rows, cols = w.shape
            assert cols % 256 == 0
            combined = {}
            for qt in TYPES:
                qb = rtn.quantize(w, qt)
                combined[qt] = decoders[qt](qb.reshape(-1), rows, cols).float()
            path = L._combined_cache_path(name, "dequant", L._tensor_hash(w), "none")
            torch.save(combined, path)

    state_dict_meta = {k: (v.untyped_storage().data_ptr(), v.numel()) for k, v in student.state_dict().items()}
    replaced = L.replace_linear_with_mixed_quant(student, TYPES)
    replaced.update(L.replace_embedding_with_mixed_quant(student, TYPES))
    targeted = {n + ".weight" for n in replaced}
    total_8bit = TR.compute_total_8bit_bytes(state_dict_meta)
    non_targeted = TR.compute_non_targeted_8bit_bytes(state_dict_meta, targeted)
    target_bytes = BUDGET * total_8bit
    for p in student.parameters():
        p.requires_grad = False
    names = sorted(replaced)

    # ---- Q8_0 teacher ---------------------------------------------------------
    teacher = fp32_model()
    tsd, meta = {}, {}
    for name, mod in teacher.named_modules():
        if isinstance(mod, (torch.nn.Linear, torch.nn.Embedding)):
            w = mod.weight.detach().numpy()
            tsd[name + ".weight"] = torch.from_numpy(
                gq.quantize(w, GGMLQuantizationType.Q8_0).reshape(-1, 34).copy())
            meta[name + ".weight"] = {"out_features": w.shape[0], "in_features": w.shape[1]}
    Q8.wrap_q8_teacher(teacher, tsd, meta)
    teacher.eval()

    # ---- inputs ----------------------------------------------------------------
    x, y = syn.random_tokens(shape, "cpu", seed=TOKEN_SEED)
    rng = np.random.default_rng(GATE_SEED)
    gates0 = {n: (rng.standard_normal(len(TYPES)) * 0.1).astype(np.float32) for n in names}
    out = {"x": x.numpy(), "y": y.numpy(), "names": np.array(names), "types": np.array(TYPES),
           "target_bytes": np.float64(target_bytes), "non_targeted_bytes": np.float64(non_targeted)}
    for n in names:
        out[f"gates0/{n}"] = gates0[n]

    with torch.no_grad():
        t_logits = teacher(input_ids=x).logits.float()

    for variant, (T, kl_w, size_w, step) in VARIANTS.items():
        trainable = []
        for n in names:
            layer = replaced[n]
            with torch.no_grad():
                layer.gates.copy_(torch.from_numpy(gates0[n]))
            layer.gates.requires_grad = True
            layer.gates.grad = None
            trainable.append(layer.gates)
        optimizer = torch.optim.AdamW(trainable, lr=LR, betas=(0.9, 0.95))
        scheduler = torch.optim.lr_scheduler.CosineAnnealingLR(optimizer, T_max=MAX_STEPS, eta_min=1e-3)
        tau = TR.anneal_temperature(step, MAX_STEPS, TEMP_START, TEMP_END)
        for layer in replaced.values():
            layer.set_temperature(tau)

        # trainer.py:2538-2575 (plain path, loss on the model's device)
        logits = student(input_ids=x).logits
        V = logits.size(-1)
        lm_loss = F.cross_entropy(logits.view(-1, V), y.view(-1))
        student_log_probs = F.log_softmax(logits / T, dim=-1)
        teacher_probs = F.softmax(t_logits / T, dim=-1)
        per_token_kl = F.kl_div(student_log_probs.view(-1, V), teacher_probs.view(-1, V),
                                reduction="none").sum(dim=-1) * (T * T)
        distill_loss = per_token_kl.mean()
        # trainer.py:2577-2590
        current_bytes = L.total_effective_bytes(replaced) + non_targeted
        size_loss = torch.relu(torch.abs(current_bytes / target_bytes - 1.0) - TOL) ** 2
        loss = lm_loss + kl_w * distill_loss + size_w * size_loss
        optimizer.zero_grad()
        loss.backward()
        grads = {n: replaced[n].gates.grad.detach().clone() for n in names}
        # trainer.py:2606-2616
        torch.nn.utils.clip_grad_norm_(trainable, max_norm=1.0)
        optimizer.step()
        scheduler.step()

        pre = f"{variant}/"
        out[pre + "args"] = np.array([T, kl_w, size_w, step], dtype=np.float64)
        out[pre + "tau"] = np.float64(tau)
        out[pre + "loss"] = np.float64(loss.item())
        out[pre + "lm_loss"] = np.float64(lm_loss.item())
        out[pre + "distill_loss"] = np.float64(distill_loss.item())
        out[pre + "size_bytes"] = np.float64(current_bytes.item())
        out[pre + "size_loss"] = np.float64(size_loss.item())
        out[pre + "logits"] = logits.detach()[0, :LOGIT_ROWS].numpy().astype(np.float32)
        for n in names:
            out[pre + f"grad/{n}"] = grads[n].numpy().astype(np.float64)
            out[pre + f"gates1/{n}"] = replaced[n].gates.detach().numpy().astype(np.float32)
        out[pre + "assign"] = np.array([replaced[n].get_assignment() for n in names])
        print(f"{variant}: loss {loss.item():.6f} (lm {lm_loss.item():.6f}, kl {distill_loss.item():.6f}, "
              f"size {size_loss.item():.3e}), tau {tau:.4f}")

    np.savez_compressed(HERE / "step_golden.npz", **out)
    print("step golden written")


if __name__ == "__main__":
    main()
