"""Generate the golden vectors in this directory from the reference itself.

Run once, in a container that has the reference checkout (it is never run by
the tests or on the GPU box):

    python tests/golden/make_golden.py --reference <path to voodoo-dyn-quant>

What it records (all seeded, all small):

* ``dequant_golden.npz`` -- seeded random valid GGUF blocks for Q8_0, Q4_K,
  Q5_K, Q6_K, IQ4_XS (decoded by the reference's torch decoders,
  ``voodoo_quant/layers.py:62-213`` and ``quants/gpu_dequant.py:460-519``) and
  for Q2_K, Q3_K (decoded by gguf-py 0.19.0, the reference's declared
  dependency; the reference has no decoder for them).  Every format is also
  cross-checked against gguf-py here.  Each format carries edge blocks whose
  fp16 scales are +0, -0, subnormal, 65504, +inf, -inf and NaN.
* ``ptqr_golden.npz`` -- the reference's per-token routed forwards
  (``_RoutedMixedLinear``, ``_MixedEmbeddingRowFunctionLazy`` with a fixed
  routing) and their straight-through backward.
* ``mixlinear_golden.npz`` -- the reference's ``_MixedWeightFunction`` +
  ``F.linear`` autograd (``layers.py:322-363``, ``:1730-1731``) in float32:
  Y, dX, d(probs) and d(gates) for seeded X, dY, gates and packed candidates.
* ``q8quant_golden.npz`` -- gguf-py 0.19.0's Q8_0 quantiser (its restatement
  of ggml's reference ``quantize_row_q8_0``, which the reference reaches
  through libggml, ``voodoo_quant/ggml.py:171-221``) on seeded float32
  weights with edge blocks: all zero, exact .5 ties, the largest float below
  1/2, signed zeros, tiny and huge magnitudes; and on the same weights
  rounded to bfloat16.  ``--only q8quant`` regenerates just this file (it
  needs gguf-py, not the reference checkout).
* ``loss_golden.npz`` -- the reference's ``_chunked_forward_loss``
  (``training/trainer.py:753-832``) on seeded logits through an identity
  head: CE, KL and the gradient with respect to the student logits.
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

FORMATS = {  # name -> (elements per block, bytes per block, fp16 scale offsets)
    "Q8_0": (32, 34, (0,)),
    "Q2_K": (256, 84, (80, 82)),
    "Q3_K": (256, 110, (108,)),
    "Q4_K": (256, 144, (0, 2)),
    "Q5_K": (256, 176, (0, 2)),
    "Q6_K": (256, 210, (208,)),
    "IQ4_XS": (256, 136, (0,)),
}

EDGE_F16 = np.array([0.0, -0.0, 2.0 ** -24, 6.097555e-05, 65504.0, np.inf, -np.inf, np.nan], dtype=np.float16)


def random_blocks(rng: np.random.Generator, fmt: str, nblocks: int, edge: bool) -> np.ndarray:
    bs, bb, offs = FORMATS[fmt]
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    for j, off in enumerate(offs):
        if edge:
            vals = EDGE_F16[(np.arange(nblocks) + 3 * j) % EDGE_F16.size]
        else:
            mag = np.exp(rng.uniform(np.log(1e-4), np.log(5e-2), size=nblocks))
            vals = (mag * rng.choice([-1.0, 1.0], size=nblocks)).astype(np.float16)
        raw[:, off:off + 2] = vals.astype(np.float16).view(np.uint8).reshape(nblocks, 2)
    return raw


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(nan | (a.view(np.uint32) == b.view(np.uint32))))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()

    scratch = tempfile.mkdtemp(prefix="vq_golden_")
    # The reference's cache module creates compile-cache dirs at import; point
    # them at scratch space so the (read-only) reference tree is untouched.
    os.environ["TRITON_CACHE_DIR"] = os.path.join(scratch, "triton")
    os.environ["TORCHINDUCTOR_CACHE_DIR"] = os.path.join(scratch, "inductor")
    sys.path.insert(0, args.reference)

    import torch
    import torch.nn.functional as F
    import gguf
    from gguf import quants as gq
    from voodoo_quant import layers as L
    from voodoo_quant.quants import gpu_dequant as GD

    torch.set_num_threads(1)
    ref_torch = {
        "Q8_0": L._dequantize_q8_0_gpu,
        "Q4_K": L._dequantize_q4_K_gpu,
        "Q5_K": L._dequantize_q5_K_gpu,
        "Q6_K": L._dequantize_q6_K_gpu,
        "IQ4_XS": GD._dequantize_iq4_xs_gpu,
    }
    gg_type = {name: getattr(gguf.GGMLQuantizationType, name) for name in FORMATS}

    rng = np.random.default_rng(20261201)
    out = {}
    rows, cols = 8, 1024
    for fmt, (bs, bb, _) in FORMATS.items():
        nb = rows * cols // bs
        regular = random_blocks(rng, fmt, nb, edge=False)
        edge = random_blocks(rng, fmt, 2 * EDGE_F16.size, edge=True)
        for tag, raw in (("regular", regular), ("edge", edge)):
            r = raw.shape[0] * bs // cols if tag == "regular" else raw.shape[0]
            c = cols if tag == "regular" else bs
            gref = gq.dequantize(raw.reshape(-1), gg_type[fmt]).reshape(-1).astype(np.float32)
            if fmt in ref_torch:
                with np.errstate(all="ignore"):
                    tref = ref_torch[fmt](torch.from_numpy(raw.reshape(-1).copy()), r, c).numpy().reshape(-1)
                if not same_bits(tref, gref):
                    raise SystemExit(f"reference torch decoder and gguf-py disagree on {fmt}/{tag}")
                expected = tref
            else:
                expected = gref
            out[f"{fmt}/{tag}/bytes"] = raw
            out[f"{fmt}/{tag}/expected"] = expected.reshape(r, c)
        print(f"{fmt}: reference decoders agree bit for bit")
    np.savez_compressed(HERE / "dequant_golden.npz", **out)

    # ---- mixture + linear, reference autograd in float32 ----------------------
    mix = {}
    for case, (fmts, T, IN, OUT, tau) in {
        "k4": (["Q4_K", "Q5_K", "Q6_K", "Q8_0"], 48, 512, 96, 1.0),
        "k5": (["Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 40, 768, 64, 0.5),
        "k6": (["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"], 24, 256, 32, 0.5),
    }.items():
        cands = []
        for k, fmt in enumerate(fmts):
            bs, bb, _ = FORMATS[fmt]
            raw = random_blocks(rng, fmt, OUT * IN // bs, edge=False)
            # keep the decoded magnitudes O(0.02) like a real weight matrix
            for off in FORMATS[fmt][2]:
                vals = (rng.uniform(5e-4, 2e-3, size=raw.shape[0]) * rng.choice([-1, 1], raw.shape[0])).astype(np.float16)
                raw[:, off:off + 2] = vals.view(np.uint8).reshape(-1, 2)
            w = gq.dequantize(raw.reshape(-1), gg_type[fmt]).reshape(OUT, IN).astype(np.float32)
            cands.append(torch.from_numpy(w))
            mix[f"{case}/cand{k}/bytes"] = raw
        x = torch.from_numpy(rng.standard_normal((T, IN)).astype(np.float32)).requires_grad_(True)
        gates = torch.from_numpy(rng.standard_normal(len(fmts)).astype(np.float32)).requires_grad_(True)
        dy = torch.from_numpy(rng.standard_normal((T, OUT)).astype(np.float32))
        probs = F.softmax(gates / tau, dim=0)
        probs.retain_grad()
        mixed = L._MixedWeightFunction.apply(torch.float32, probs, *cands)
        y = F.linear(x, mixed)
        y.backward(dy)
        mix[f"{case}/formats"] = np.array(fmts)
        mix[f"{case}/tau"] = np.float32(tau)
        mix[f"{case}/x"] = x.detach().numpy()
        mix[f"{case}/dy"] = dy.numpy()
        mix[f"{case}/gates"] = gates.detach().numpy()
        mix[f"{case}/y"] = y.detach().numpy()
        mix[f"{case}/dx"] = x.grad.numpy()
        mix[f"{case}/dprobs"] = probs.grad.numpy()
        mix[f"{case}/dgates"] = gates.grad.numpy()
    np.savez_compressed(HERE / "mixlinear_golden.npz", **mix)
    print("mixlinear golden written")

    # ---- chunked CE + KL loss through an identity head ------------------------
    from types import SimpleNamespace
    from voodoo_quant.training import trainer as TR

    torch.cuda.synchronize = lambda *a, **k: None  # the reference fences CUDA per chunk

    class _Base(torch.nn.Module):
        def __init__(self, logits):
            super().__init__()
            self.logits = torch.nn.Parameter(logits)

        def forward(self, input_ids):
            return SimpleNamespace(last_hidden_state=self.logits * 1.0)

    class _Model(torch.nn.Module):
        def __init__(self, logits):
            super().__init__()
            self.model = _Base(logits)
            self.lm_head = torch.nn.Identity()

    loss = {}
    for case, (B, S, V, temp, chunk) in {
        "t1": (2, 8, 1000, 1.0, 5),
        "t2": (3, 5, 777, 2.0, 4),
    }.items():
        s = torch.from_numpy((rng.standard_normal((B, S, V)) * 3).astype(np.float32))
        t = torch.from_numpy((rng.standard_normal((B, S, V)) * 3).astype(np.float32))
        y = torch.from_numpy(rng.integers(0, V, size=(B, S)).astype(np.int64))
        student, teacher = _Model(s.clone()), _Model(t.clone())
        teacher.requires_grad_(False)
        lm, kl = TR._chunked_forward_loss(student, teacher, torch.zeros(B, S, dtype=torch.long), y, temp,
                                          chunk=chunk, loss_device="cpu", teacher_device="cpu")
        loss[f"{case}/student"] = s.numpy()
        loss[f"{case}/teacher"] = t.numpy()
        loss[f"{case}/targets"] = y.numpy()
        loss[f"{case}/temperature"] = np.float32(temp)
        loss[f"{case}/ce"] = np.float64(lm)
        loss[f"{case}/kl"] = np.float64(kl)
        loss[f"{case}/dlogits"] = student.model.logits.grad.numpy()
    np.savez_compressed(HERE / "loss_golden.npz", **loss)
    print("loss golden written")

    # ---- PTQR (per-token routing) forward with the straight-through backward --
    # A fixed routing stands in for the Gumbel sample so that the B200 path
    # can be run on the same routing.
    prng = np.random.default_rng(20261201)
    ptqr = {}
    fmts = ["Q4_K", "Q5_K", "Q6_K", "Q8_0"]
    T, IN, OUT, tau = 40, 512, 64, 1.0
    cands = []
    for k, fmt in enumerate(fmts):
        bs, bb, _ = FORMATS[fmt]
        raw = random_blocks(prng, fmt, OUT * IN // bs, edge=False)
        for off in FORMATS[fmt][2]:
            vals = (prng.uniform(5e-4, 2e-3, size=raw.shape[0]) * prng.choice([-1, 1], raw.shape[0])).astype(np.float16)
            raw[:, off:off + 2] = vals.view(np.uint8).reshape(-1, 2)
        cands.append(torch.from_numpy(gq.dequantize(raw.reshape(-1), gg_type[fmt]).reshape(OUT, IN).astype(np.float32)))
        ptqr[f"lin/cand{k}/bytes"] = raw
    x = torch.from_numpy(prng.standard_normal((T, IN)).astype(np.float32)).requires_grad_(True)
    gates = torch.from_numpy(prng.standard_normal(len(fmts)).astype(np.float32)).requires_grad_(True)
    dy = torch.from_numpy(prng.standard_normal((T, OUT)).astype(np.float32))
    routing = torch.from_numpy(prng.integers(0, len(fmts), size=T).astype(np.int64))
    probs = F.softmax(gates / tau, dim=0)
    probs.retain_grad()
    y = L._RoutedMixedLinear.apply(torch.float32, probs, routing, x, *cands)
    y.backward(dy)
    ptqr["lin/formats"] = np.array(fmts)
    ptqr["lin/tau"] = np.float32(tau)
    ptqr["lin/x"] = x.detach().numpy()
    ptqr["lin/dy"] = dy.numpy()
    ptqr["lin/gates"] = gates.detach().numpy()
    ptqr["lin/routing"] = routing.numpy()
    ptqr["lin/y"] = y.detach().numpy()
    ptqr["lin/dx"] = x.grad.numpy()
    ptqr["lin/dprobs"] = probs.grad.numpy()
    ptqr["lin/dgates"] = gates.grad.numpy()

    V, D = 64, 512
    qbytes = []
    for k, fmt in enumerate(fmts):
        bs, bb, _ = FORMATS[fmt]
        raw = random_blocks(prng, fmt, V * D // bs, edge=False)
        for off in FORMATS[fmt][2]:
            vals = (prng.uniform(5e-4, 2e-3, size=raw.shape[0]) * prng.choice([-1, 1], raw.shape[0])).astype(np.float16)
            raw[:, off:off + 2] = vals.view(np.uint8).reshape(-1, 2)
        qbytes.append(torch.from_numpy(raw.copy()))
        ptqr[f"emb/cand{k}/bytes"] = raw
    row_ids = torch.from_numpy(np.sort(prng.choice(V, size=20, replace=False)).astype(np.int64))
    eroute = torch.from_numpy(prng.integers(0, len(fmts), size=20).astype(np.int64))
    egates = torch.from_numpy(prng.standard_normal(len(fmts)).astype(np.float32)).requires_grad_(True)
    eprobs = F.softmax(egates, dim=0)
    eprobs.retain_grad()
    rows_out = L._MixedEmbeddingRowFunctionLazy.apply(torch.bfloat16, tuple(fmts), V, D, D, eprobs, eroute, row_ids,
                                                      *qbytes)
    G = torch.from_numpy(prng.standard_normal((20, D)).astype(np.float32))
    rows_out.float().backward(G)
    ptqr["emb/row_ids"] = row_ids.numpy()
    ptqr["emb/routing"] = eroute.numpy()
    ptqr["emb/gates"] = egates.detach().numpy()
    ptqr["emb/grad_out"] = G.numpy()
    ptqr["emb/rows"] = rows_out.detach().float().numpy()
    ptqr["emb/dprobs"] = eprobs.grad.numpy()
    np.savez_compressed(HERE / "ptqr_golden.npz", **ptqr)
    print("ptqr golden written")


def make_q8quant_golden() -> None:
    import torch
    from gguf import GGMLQuantizationType, quants

    rng = np.random.default_rng(7)
    w = (rng.standard_normal((24, 256)) * np.exp(rng.normal(0.0, 2.0, (24, 1)))).astype(np.float32)
    w[0, :32] = 0.0
    ties = np.array([127.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, np.nextafter(np.float32(0.5), np.float32(0)),
                     -np.nextafter(np.float32(0.5), np.float32(0)), 126.5, -126.5, 63.5, 0.0, -0.0, 3.4999998, 1.0],
                    dtype=np.float32)
    w[1, :16] = ties
    w[1, 16:32] = -ties
    w[2, :32] = rng.standard_normal(32).astype(np.float32) * np.float32(1e-30)
    w[3, :32] = rng.standard_normal(32).astype(np.float32) * np.float32(1e30)
    w[4, :32] = -0.0
    wb = torch.from_numpy(w).to(torch.bfloat16).float().numpy()
    q = quants.quantize(w, GGMLQuantizationType.Q8_0).reshape(-1, 34)
    qb = quants.quantize(wb, GGMLQuantizationType.Q8_0).reshape(-1, 34)
    np.savez_compressed(HERE / "q8quant_golden.npz", w=w, q=q, w_bf16=wb, q_bf16=qb)
    print("q8quant golden written")


if __name__ == "__main__":
    if "--only" in sys.argv and sys.argv[sys.argv.index("--only") + 1] == "q8quant":
        make_q8quant_golden()
    else:
        main()
        make_q8quant_golden()
