"""Benchmark of the gated-candidate distillation step on B200.

Default workload (the configuration the metric
"gated-distill train tokens/s at 1/2/4/8 B200" is quoted on): the full
distillation step of a random-init 8B Llama-3-shape decoder -- 32 layers,
hidden 4096, 32 query / 8 KV heads, SwiGLU 14336, vocabulary 128256, untied
-- whose every Linear and the embedding are gated over K = 6 packed
candidates (Q2_K ... Q8_0), against a Q8_0 teacher of the same weights;
batch 4 x seq 4096 = 16384 tokens per step, loss CE + 1.0 KL, size budget
30 %.  A step is the reference's step loop (voodoo_quant/training/trainer.py:
2443-2666): student forward, teacher forward, fused loss, size term,
backward, gate all-reduce, clip, AdamW, cosine LR.  Candidates come from the
round-to-nearest GGUF packer (libggml is unavailable); weights and tokens are
seeded synthetic draws.

--gpus N (torchrun, one process per GPU): both models tensor-parallel over
the N GPUs (Llama adapter); every rank runs the same batch, total work is
fixed ("strong" scaling); value = tokens / max-over-ranks step time.

The line also carries ``mix_gemm``: the metric's second half, the fused
mix-GEMM kernels of BASELINE.json configs[1] (one gated Linear X [8192 x 4096],
W [14336 x 4096], K = 5) as fractions of the measured bf16 peak, timed on
rank 0's GPU in the same run.  ``--workload layer`` makes that layer the
whole benchmark.

--impl reference: the reference's algorithm on the host cores (the float32
numpy port of its torch CPU path, layers.py:322-363 + F.linear), on a bounded
sample of the same workload, reported in the same unit (see run_reference).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "voodoo-dyn-quant_b200"))

T_TOK, N_OUT, K_IN = 8192, 14336, 4096
TYPES = ["Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]
TAU = 0.5
METRIC = "gated-distill train tokens/s"
LAYER_METRIC = "gated-Linear fwd + dX + gate-grad tokens/s (config 2)"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# dram__bytes_read.sum + dram__bytes_write.sum per launch of each config-2 GEMM
# at full size on one B200, from a single-pass ncu capture of this benchmark
NCU_TRAFFIC_BYTES = {"fwd": 818.1e6, "dx": 1032.6e6, "gategrad": 1115.4e6}
BPW = {"Q2_K": 84 / 256, "Q3_K": 110 / 256, "Q4_K": 144 / 256, "Q5_K": 176 / 256, "Q6_K": 210 / 256,
       "Q8_0": 34 / 32, "IQ4_XS": 136 / 256}
WORKLOAD_NAMES = {
    "tiny": "config1: tiny Llama gated distillation step",
    "0.6b": "config3: ~0.6B dense decoder gated distillation step",
    "8b": "config4: 8B Llama-3-shape gated distillation step",
    "32b": "config5: 32B-shape dense decoder gated distillation step",
}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def layer_config(n_gpus: int, extra=None):
    c = {
        "workload": "config2: gated Linear X[8192x4096] W[14336x4096], K=5 {Q3_K,Q4_K,Q5_K,Q6_K,Q8_0}, "
                    "tau=0.5, fwd+dX+gate-grad",
        "tokens_per_step": T_TOK,
        "candidates": TYPES,
        "parallelism": f"tp{n_gpus}" if n_gpus > 1 else "tp1",
        "l2": "inputs larger than L2 (X 67 MB, dY 235 MB, packed candidates 209 MB, W_mix 117 MB)",
    }
    if extra:
        c.update(extra)
    return c


def step_config(workload: str, shape, world: int) -> dict:
    """The step workload's description: a function of the workload and N only,
    so both arms print the same object."""
    return {"workload": WORKLOAD_NAMES.get(workload, workload), "layers": shape.layers, "hidden": shape.hidden,
            "heads": shape.heads, "kv_heads": shape.kv_heads, "ffn": shape.ffn, "vocab": shape.vocab,
            "tied": shape.tied, "batch": shape.batch, "seq": shape.seq, "tokens_per_step": shape.batch * shape.seq,
            "candidates": shape.candidates, "attention_candidates": shape.attention_candidates,
            "row_scale_sigma": shape.row_scale_sigma, "budget": shape.budget, "loss": "CE + 1.0 * T^2 KL, T = 1",
            "parallelism": f"tp{world}",
            "l2": "activations, logits and packed candidates far larger than L2"}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling (200 ms) started before the timed region; summary()
    keeps the samples whose timestamps fall inside [mark_start, mark_end]."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        deadline = time.time() + 5.0   # wait for the first sample so the timed region is covered
        while self.proc is not None and time.time() < deadline and os.path.getsize(self.path) == 0:
            time.sleep(0.05)
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()
        time.sleep(0.25)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        from datetime import datetime

        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    ts = datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    continue
                rows.append((ts, f))
            os.unlink(self.path)
        inside = [f for ts, f in rows if self.t0 is not None and self.t0 - 0.2 <= ts <= (self.t1 or ts) + 0.2]
        use = inside or [f for _, f in rows]

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = sorted(v for v in (num(f[2]) for f in use) if v is not None)
        mx = [v for v in (num(f[3]) for f in use) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for f in use for i in range(4) if f[5 + i].lower().startswith("active")})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(inside), "samples_total": len(rows)}


# ----------------------------------------------------------------------------- config-2 layer
def make_layer(device, rank=0, world=1):
    import torch
    from voodoo_quant.layers import MixedQuantLinear
    from voodoo_quant.parallel import ShardSpec, block_aligned_split
    from voodoo_quant.quants import rtn

    g = torch.Generator(device=device).manual_seed(0)
    w = torch.randn(N_OUT, K_IN, device=device, generator=g) * 0.02
    full = {q: rtn.quantize(w, q) for q in TYPES}
    gates = torch.randn(len(TYPES), generator=torch.Generator().manual_seed(1))
    if world > 1:
        off, n = block_aligned_split(N_OUT, world, rank)
        spec = ShardSpec(full_out=N_OUT, full_in=K_IN, row_offset=off, row_len=n)
        layer = MixedQuantLinear(K_IN, n, TYPES, w[off:off + n], tensor_name="bench.proj", shard_spec=spec,
                                 candidate_bytes=full)
    else:
        layer = MixedQuantLinear(K_IN, N_OUT, TYPES, w, tensor_name="bench.proj", candidate_bytes=full)
    del w, full
    with torch.no_grad():
        layer.gates.copy_(gates)
    layer.set_temperature(TAU)
    return layer


def make_inputs(device, n_out_local, seed=2):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(T_TOK, K_IN, device=device, generator=g)
    ch = torch.randperm(K_IN, generator=torch.Generator().manual_seed(3))[: K_IN // 100].to(device)
    x[:, ch] *= 20.0
    x = x.to(torch.bfloat16)
    dy = torch.randn(T_TOK, n_out_local, device=device, generator=g).to(torch.bfloat16)
    return x, dy


def time_layer_kernels(layer, x, dy, iters: int) -> dict:
    """Average CUDA-event time (ms) of each kernel of the layer step, launched
    back to back on the current stream: mix, forward GEMM, dX GEMM, gate-grad
    GEMM (inputs larger than L2, so each launch streams from HBM)."""
    import torch
    from voodoo_quant import _C

    stream = torch.cuda.current_stream()
    n_loc = layer.out_features
    blocks = layer._candidate_blocks()
    probs = layer.get_probs().detach()
    pad = layer.padded_in_features
    ws = layer._gategrad_workspace(x.device)
    wm = _C.mix(TYPES, blocks, probs, n_loc, pad, K_IN)
    names = ["mix", "fwd", "dx", "gategrad"]
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(iters)]
    for i in range(iters + 2):
        e = evs[i - 2] if i >= 2 else None
        if e: e[0].record(stream)
        _C.mix(TYPES, blocks, probs, n_loc, pad, K_IN, out=wm)
        if e: e[1].record(stream)
        _C.linear_fwd(x, wm, n_loc, K_IN)
        if e: e[2].record(stream)
        _C.linear_dx(dy, wm, K_IN)
        if e: e[3].record(stream)
        _C.gategrad(dy, x, TYPES, blocks, n_loc, K_IN, pad, workspace=ws)
        if e: e[4].record(stream)
    torch.cuda.synchronize()
    return {n: sum(e[j].elapsed_time(e[j + 1]) for e in evs) / len(evs) for j, n in enumerate(names)}


def layer_kernel_summary(kt: dict, n_loc: int) -> dict:
    """Per-kernel TFLOP/s (GEMMs: 2 T N Kin each) or GB/s (mix: packed bytes
    read + bf16 W_mix written) and fractions of the measured burst peaks."""
    pk, pk_kind = peaks()
    peak_t = float(pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    peak_b = float(pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    flops_gemm = 2.0 * T_TOK * n_loc * K_IN
    ach = {n: flops_gemm / (kt[n] * 1e-3) / 1e12 for n in ("fwd", "dx", "gategrad")}
    mix_bytes = n_loc * K_IN * sum(BPW[q] for q in TYPES) + n_loc * K_IN * 2
    kernels = {n: {"ms": round(kt[n], 4), "TFLOP/s": round(ach[n], 1), "frac": round(ach[n] / peak_t, 4)}
               for n in ("fwd", "dx", "gategrad")}
    kernels["mix"] = {"ms": round(kt["mix"], 4), "GB/s": round(mix_bytes / (kt["mix"] * 1e-3) / 1e9, 1),
                      "frac": round(mix_bytes / (kt["mix"] * 1e-3) / 1e9 / peak_b, 4),
                      "algorithmic_bytes": int(mix_bytes)}
    gemm_ms = kt["fwd"] + kt["dx"] + kt["gategrad"]
    all_ms = gemm_ms + kt["mix"]
    return {"kernels": kernels, "peak_tflops": peak_t, "peak_gbs": peak_b,
            "peak_source": f"{pk_kind} bf16_tflops / hbm_gbs (burst)",
            "mix_gemm_frac": round(3 * flops_gemm / (gemm_ms * 1e-3) / 1e12 / peak_t, 4),
            "mix_gemm_with_mix_frac": round(3 * flops_gemm / (all_ms * 1e-3) / 1e12 / peak_t, 4),
            "ach": ach}


def layer_kernel_fractions(dev, iters: int = 10) -> dict:
    """The metric's second half on this GPU: the config-2 gated Linear's
    kernels (mix, forward, dX, gate-grad GEMMs) as fractions of the measured
    bf16 / HBM peaks; the layer is freed afterwards."""
    import torch

    layer = make_layer(dev)
    x, dy = make_inputs(dev, N_OUT)
    kt = time_layer_kernels(layer, x, dy, iters)
    s = layer_kernel_summary(kt, N_OUT)
    del layer, x, dy
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    s.pop("ach")
    s["workload"] = layer_config(1)["workload"]
    s["gemm_flops_each"] = 2.0 * T_TOK * N_OUT * K_IN
    return s


# ----------------------------------------------------------------------------- GPU arm: config-2 layer
def run_gpu(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        from voodoo_quant import parallel

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
        parallel.adopt_process_group(local)
        # the dX all-reduce runs on a second communicator whose CTAs fit on
        # the SMs the gate-gradient GEMM (and later dX chunks) leave free
        parallel.enable_input_grad_overlap(args.overlap_sms)
    from voodoo_quant import _C
    from voodoo_quant.parallel import all_reduce_gate_grads

    _C.load_library()
    layer = make_layer(dev, rank, world)
    n_loc = layer.out_features
    x, dy = make_inputs(dev, n_loc, seed=2 + rank)
    stream = torch.cuda.current_stream()

    if world > 1:
        import voodoo_quant.layers as _layers

        layer.reduce_input_grad = True  # dX all-reduce overlapped with the gate-gradient GEMM
        _layers.INPUT_GRAD_CHUNKS = args.dx_chunks

    def step(xin, dyin):
        xg = xin.requires_grad_(True) if not xin.requires_grad else xin
        y = layer(xg)
        layer.gates.grad = None
        torch.autograd.backward(y, dyin)
        if world > 1:
            all_reduce_gate_grads([layer.gates])
        return xg

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        x.grad = None
        step(x, dy)
    torch.cuda.synchronize()
    barrier()

    # The timed steps replay one CUDA graph of the step (forward, backward and
    # the TP collectives), so host launch overhead stays out of the GPU
    # timeline; every rank uses the graph only if every rank captured it.
    graph, graph_note = None, "off"
    if not args.no_graph:
        try:
            side = torch.cuda.Stream(dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                for _ in range(2):
                    x.grad = None
                    step(x, dy)
            stream.wait_stream(side)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            x.grad = None
            with torch.cuda.graph(g):
                step(x, dy)
            graph, graph_note = g, "cuda graph of the step"
            del g
        except Exception as e:  # capture unsupported here: time the eager step
            graph, graph_note = None, f"eager (capture failed: {type(e).__name__})"
        ok = torch.tensor([1.0 if graph is not None else 0.0], device=dev)
        if world > 1:
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if ok.item() < 1.0:
            graph = None
            if graph_note.startswith("cuda graph"):
                graph_note = "eager (another rank could not capture)"
        torch.cuda.synchronize()
        barrier()

    def timed_step():
        if graph is not None:
            graph.replay()
        else:
            x.grad = None
            step(x, dy)

    for _ in range(args.warmup):
        timed_step()
    torch.cuda.synchronize()
    barrier()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local).start()
    barrier()
    torch.cuda.synchronize()
    clk.mark_start()
    ev0.record(stream)
    for _ in range(args.steps):
        timed_step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk.mark_end()
    barrier()
    clk.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    clocks = clk.summary()
    assert _C.device_error() == 0

    # ---- per-kernel breakdown (same stream, CUDA events per launch) ----
    kt = time_layer_kernels(layer, x, dy, args.kernel_iters)

    # ---- e2e through the public API with host buffers ----
    # Every step copies its X and dY from pinned host memory and reads the
    # gate gradient back; the copy of step i+1 runs on a side stream while
    # step i computes (double-buffered device inputs).
    xh = x.detach().cpu().pin_memory()
    dyh = dy.cpu().pin_memory()
    gh = torch.empty(len(TYPES), dtype=torch.float32).pin_memory()
    copy_stream = torch.cuda.Stream(dev)
    xb = [torch.empty_like(x) for _ in range(2)]
    dyb = [torch.empty_like(dy) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    for b in range(2):
        free[b].record(stream)

    def issue_copy(i):
        b = i & 1
        with torch.cuda.stream(copy_stream), torch.no_grad():
            copy_stream.wait_event(free[b])
            xb[b].copy_(xh, non_blocking=True)
            dyb[b].copy_(dyh, non_blocking=True)
            ready[b].record(copy_stream)

    total = args.warmup + args.e2e_steps
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    for i in range(total):
        if i == args.warmup:
            torch.cuda.synchronize()
            barrier()
            e0.record(stream)
        b = i & 1
        if i == 0 or i == args.warmup:  # the first timed step copies inside the timed region
            issue_copy(i)
        if i + 1 < total and i + 1 != args.warmup:
            issue_copy(i + 1)
        stream.wait_event(ready[b])
        xin = xb[b]
        xin.grad = None
        step(xin, dyb[b])
        gh.copy_(layer.gates.grad, non_blocking=True)
        free[b].record(stream)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / args.e2e_steps], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())

    if rank == 0:
        s = layer_kernel_summary(kt, n_loc)
        ach, peak_t = s["ach"], s["peak_tflops"]
        dom = max(("fwd", "dx", "gategrad"), key=lambda n: kt[n])
        flops_gemm = 2.0 * T_TOK * n_loc * K_IN
        out = {
            "metric": LAYER_METRIC,
            "value": round(T_TOK / (ms * 1e-3), 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded; candidates from the round-to-nearest GGUF packer)",
            "config": layer_config(world),
            "run": {"timed_step": graph_note, "dx_allreduce_overlap_sms": args.overlap_sms if world > 1 else 0,
                    "dx_chunks": args.dx_chunks if world > 1 else 1},
            "roofline": {
                "bound": "tensor",
                "kernel": f"gemm_{dom}",
                "achieved": round(ach[dom], 1),
                "peak": peak_t,
                "unit": "TFLOP/s",
                "frac": round(ach[dom] / peak_t, 4),
                "peak_source": s["peak_source"],
                "traffic": NCU_TRAFFIC_BYTES[dom] if world == 1 else None,
                "traffic_unit": "bytes per launch (ncu dram read+write, full size)",
                "mix_gemm_frac": s["mix_gemm_frac"],
                "step_frac": round(3 * flops_gemm / (ms * 1e-3) / 1e12 / peak_t, 4),
            },
            "kernels": s["kernels"],
            "e2e": {
                "value": round(T_TOK / (e2e_ms * 1e-3), 1),
                "unit": "tokens/s",
                "h2d_bytes_per_step": int(x.numel() * 2 + dy.numel() * 2),
                "d2h_bytes_per_step": int(gh.numel() * 4),
            },
            "gpu_launches": 5 * args.steps,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = layer_cpu_baseline(args.cpu_tokens, repeats=1)
        print(json.dumps(out), flush=True)
    graph = None  # the captured graph holds NCCL work: release it before the process group
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------- host (reference algorithm)
def _host_threads() -> int:
    return os.cpu_count() or 1


def _layer_host_setup(t_sample: int):
    import numpy as np
    import torch

    sys.path.insert(0, str(ROOT))
    from oracle import mixgemm
    from voodoo_quant.quants import rtn

    torch.manual_seed(0)
    w = torch.randn(N_OUT, K_IN) * 0.02
    blocks = [rtn.quantize(w, q).numpy() for q in TYPES]
    del w
    threads = _host_threads()
    cands = mixgemm.decode_candidates(blocks, TYPES, N_OUT, K_IN, K_IN, threads=threads)  # untimed (cached _w_k)
    rng = np.random.default_rng(2)
    x = rng.standard_normal((t_sample, K_IN), dtype=np.float32)
    x[:, rng.permutation(K_IN)[: K_IN // 100]] *= 20.0
    dy = rng.standard_normal((t_sample, N_OUT), dtype=np.float32)
    gates = torch.randn(len(TYPES), generator=torch.Generator().manual_seed(1)).numpy()
    return mixgemm, cands, x, dy, gates


def _layer_host_step(mixgemm, cands, x, dy, gates):
    threads = _host_threads()
    p = mixgemm.softmax_probs(gates, TAU)
    wm = mixgemm.mixed_weight(cands, p, threads=threads)
    mixgemm.linear_fwd(x, wm)
    mixgemm.linear_dx(dy, wm)
    g = mixgemm.prob_grad(dy, x, cands, threads=threads)
    return mixgemm.gate_grad(p, g, TAU)


def layer_cpu_baseline(t_sample: int, repeats: int = 1):
    cores = _host_threads()
    mixgemm, cands, x, dy, gates = _layer_host_setup(t_sample)
    _layer_host_step(mixgemm, cands, x, dy, gates)
    t0 = time.perf_counter()
    for _ in range(repeats):
        _layer_host_step(mixgemm, cands, x, dy, gates)
    dt = (time.perf_counter() - t0) / repeats
    return {"value": round(t_sample / dt, 2), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{t_sample} of 8192 tokens of the config-2 layer (full N, Kin, K=5), float32 numpy "
                      f"(BLAS threads = {cores}); candidates pre-decoded like the reference's cached _w_k; "
                      f"value = sample tokens / measured sample time"}


def layer_linear_shapes(shape) -> list[tuple[str, int, int, list[str]]]:
    """(role, out_features, in_features, candidate menu) of one decoder layer's
    seven gated Linears (q, k, v, o, gate, up, down)."""
    hd = shape.head_dim or shape.hidden // shape.heads
    h, f = shape.hidden, shape.ffn
    att = shape.attention_candidates or shape.candidates
    mlp = shape.non_attention_candidates or shape.candidates
    return [("q_proj", shape.heads * hd, h, att), ("k_proj", shape.kv_heads * hd, h, att),
            ("v_proj", shape.kv_heads * hd, h, att), ("o_proj", h, shape.heads * hd, att),
            ("gate_proj", f, h, mlp), ("up_proj", f, h, mlp), ("down_proj", h, f, mlp)]


def gated_linear_params(shape) -> float:
    """Weights of every gated Linear of the step's student (layers + head)."""
    p_layer = sum(o * i for _, o, i, _ in layer_linear_shapes(shape))
    return float(shape.layers * p_layer + (0 if shape.tied else shape.vocab * shape.hidden))


class HostLayerSample:
    """A bounded host sample of a distillation-step workload: one decoder
    layer's seven gated Linears at the workload's shapes and menus, each
    stepped as the reference's float32 torch CPU path does it (cached
    decoded candidates W_k; W_mix = sum_k p_k W_k; Y = X W_mix^T;
    dX = dY W_mix; dW = dY^T X materialised; g_k = <dW, W_k>; softmax
    backward to the gates -- voodoo_quant/layers.py:322-363 and F.linear's
    autograd), in the oracle's numpy port, on ``tokens`` tokens.

    Each step's time splits into per-weight work (the mixture and the K
    reductions over dW, done once per tensor per step whatever the batch) and
    per-token work (the three GEMMs).  ``full_step_s`` scales the first by the
    student's gated weights over the layer's and the second by the whole
    step's algorithmic FLOPs (step_flops_per_token x tokens per step) over
    the sample's: the host's time for the full step at the rates this sample
    measured.  Attention, the loss and the teacher's per-step Q8_0 decode then
    run at GEMM speed or not at all, which flatters the host.

    Candidate values are seeded normal draws (scaled copies of one draw per
    tensor): the timed arithmetic does not depend on them, and decoding a
    layer's 1.3 G candidate weights through the oracle decoders would take
    longer than the whole timed run."""

    def __init__(self, shape, tokens: int, seed: int = 0):
        import numpy as np

        sys.path.insert(0, str(ROOT))
        from oracle import mixgemm

        self.mixgemm = mixgemm
        self.shape, self.tokens = shape, tokens
        self.threads = _host_threads()
        rng = np.random.default_rng(seed)
        self.tensors = []
        self.p_layer = 0
        for role, n_out, n_in, types in layer_linear_shapes(shape):
            base = rng.standard_normal((n_out, n_in), dtype=np.float32)
            base *= np.float32(0.02)
            cands = [base * np.float32(1.0 + 0.01 * k) for k in range(len(types))]
            del base
            gates = rng.standard_normal(len(types)).astype(np.float32)
            x = rng.standard_normal((tokens, n_in), dtype=np.float32)
            dy = rng.standard_normal((tokens, n_out), dtype=np.float32)
            self.tensors.append((role, cands, gates, x, dy))
            self.p_layer += n_out * n_in

    def step(self) -> tuple[float, float]:
        """One step of every tensor; returns (per-weight s, per-token s)."""
        mg, th = self.mixgemm, self.threads
        w_s = t_s = 0.0
        for _, cands, gates, x, dy in self.tensors:
            t0 = time.perf_counter()
            p = mg.softmax_probs(gates, 1.0)
            wm = mg.mixed_weight(cands, p, threads=th)
            t1 = time.perf_counter()
            mg.linear_fwd(x, wm)
            mg.linear_dx(dy, wm)
            dw = dy.T @ x
            t2 = time.perf_counter()
            g = mg.prob_grad_from_dw(dw, cands, threads=th)
            mg.gate_grad(p, g, 1.0)
            t3 = time.perf_counter()
            w_s += (t1 - t0) + (t3 - t2)
            t_s += t2 - t1
        return w_s, t_s

    def full_step_s(self, w_s: float, t_s: float) -> float:
        fpt = step_flops_per_token(self.shape)
        step_tokens = self.shape.batch * self.shape.seq
        sample_flops = 6.0 * self.p_layer * self.tokens
        return w_s * gated_linear_params(self.shape) / self.p_layer + t_s * fpt * step_tokens / sample_flops

    def describe(self) -> str:
        return (f"one decoder layer of the workload (7 gated Linears, {self.p_layer / 1e6:.0f} M weights, "
                f"K = {len(self.shape.candidates)}) on {self.tokens} tokens per step: mixture, forward, dX, "
                f"dW and the K reductions, float32 numpy on {self.threads} threads; full-step time = per-weight "
                f"time x {gated_linear_params(self.shape) / self.p_layer:.1f} (student gated weights / layer's) "
                f"+ per-token time x step FLOPs / sample FLOPs "
                f"({step_flops_per_token(self.shape) / 1e9:.2f} GFLOP/token x {self.shape.batch * self.shape.seq} "
                f"tokens); attention, loss and teacher decode counted at GEMM speed")


def step_cpu_baseline(shape, tokens: int = 256, repeats: int = 2) -> dict:
    """The full step's host baseline from HostLayerSample (rank 0, N = 1)."""
    s = HostLayerSample(shape, tokens)
    s.step()
    w = t = 0.0
    for _ in range(repeats):
        a, b = s.step()
        w, t = w + a, t + b
    full = s.full_step_s(w / repeats, t / repeats)
    return {"value": round(shape.batch * shape.seq / full, 4), "unit": "tokens/s", "cores": s.threads,
            "kind": "port", "sample_ms_per_step": round((w + t) / repeats * 1e3, 1),
            "full_step_s_estimate": float(f"{full:.4g}"), "sample": s.describe()}


def run_reference(args):
    """The reference arm: the reference's algorithm on the host cores (the
    oracle's float32 numpy port; the reference itself is Python and does not
    travel to the GPU box), rank 0 only, on the same workload, config, metric
    and unit as the GPU arm.

    * step workloads (default 8b): each step is one HostLayerSample step
      (one decoder layer on ``--cpu-tokens`` tokens, timed as it runs);
      ``ms_per_step`` is that measured time, ``value`` the full step's tokens
      over the full-step time those rates give (HostLayerSample.full_step_s).
    * layer: each step is the full config-2 layer step, all 8192 tokens.
    """
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    cores = _host_threads()
    if args.workload == "layer":
        mixgemm, cands, x, dy, gates = _layer_host_setup(T_TOK)
        for _ in range(args.warmup):
            _layer_host_step(mixgemm, cands, x, dy, gates)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            _layer_host_step(mixgemm, cands, x, dy, gates)
        dt = (time.perf_counter() - t0) / args.steps
        v = round(T_TOK / dt, 2)
        metric, cfg, ms = LAYER_METRIC, layer_config(world), dt * 1e3
        sample = "the full config-2 layer step (8192 tokens) per step, float32 numpy restatement of the " \
                 "reference's torch CPU path, candidates pre-decoded like its cached _w_k"
        extra = {}
    else:
        from voodoo_quant.training import synthetic as S

        shape = S.SHAPES[args.workload]
        s = HostLayerSample(shape, args.cpu_tokens)
        for _ in range(args.warmup):
            s.step()
        w = t = 0.0
        t0 = time.perf_counter()
        for _ in range(args.steps):
            a, b = s.step()
            w, t = w + a, t + b
        dt = (time.perf_counter() - t0) / args.steps
        full = s.full_step_s(w / args.steps, t / args.steps)
        v = round(shape.batch * shape.seq / full, 4)
        metric, cfg, ms = METRIC, step_config(args.workload, shape, world), dt * 1e3
        sample = s.describe()
        extra = {"full_step_s_estimate": float(f"{full:.4g}"), "sample_tokens_per_step": args.cpu_tokens}
    out = {
        "metric": metric, "value": v, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)", "config": cfg, "impl": "reference",
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample, **extra},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def run_ncu_case():
    """One launch each of the mix, forward GEMM, gate-gradient and loss kernels
    at sizes an ncu --set full capture finishes quickly (inputs still larger
    than L2): config-2 candidates, GEMMs at T=4096, loss 1024 x 128256."""
    import torch
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(N_OUT, K_IN, device=dev, generator=g) * 0.02
    blocks = [rtn.quantize(w, q) for q in TYPES]
    del w
    probs = torch.softmax(torch.randn(len(TYPES), device=dev, generator=g), 0)
    wm = _C.mix(TYPES, blocks, probs, N_OUT, K_IN, K_IN)
    x = torch.randn(4096, K_IN, device=dev, generator=g).to(torch.bfloat16)
    dy = torch.randn(4096, N_OUT, device=dev, generator=g).to(torch.bfloat16)
    _C.linear_fwd(x, wm, N_OUT, K_IN)
    _C.gategrad(dy, x, TYPES, blocks, N_OUT, K_IN, K_IN)
    V, R = 128256, 1024
    s = (torch.randn(R, V, device=dev, generator=g) * 3).to(torch.bfloat16)
    t = (torch.randn(R, V, device=dev, generator=g) * 3).to(torch.bfloat16)
    y = torch.randint(0, V, (R,), device=dev, generator=g)
    _C.loss_fused(s, t, y, 1.0, 1.0 / R, 1.0 / R)
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    print("ncu case ok", flush=True)


def run_ncu_case_tp8():
    """One launch each of the forward, dX and gate-gradient GEMMs at two TP-8
    shard shapes of the 8B step (T = 16384): q_proj (N = 512, Kin = 4096) and
    o_proj (N = 4096, Kin = 512), six candidates -- the small-shard GEMMs
    whose fixed per-tile costs dominate at TP-8."""
    import torch
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    types = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]
    T = 16384
    for n, kin in ((512, 4096), (4096, 512)):
        w = torch.randn(n, kin, device=dev, generator=g) * 0.02
        blocks = [rtn.quantize(w, q) for q in types]
        probs = torch.softmax(torch.randn(len(types), device=dev, generator=g), 0)
        wm = _C.mix(types, blocks, probs, n, kin, kin)
        x = torch.randn(T, kin, device=dev, generator=g).to(torch.bfloat16)
        dy = torch.randn(T, n, device=dev, generator=g).to(torch.bfloat16)
        _C.linear_fwd(x, wm, n, kin)
        _C.linear_dx(dy, wm, kin)
        _C.gategrad(dy, x, types, blocks, n, kin, kin)
    torch.cuda.synchronize()
    assert _C.device_error() == 0
    print("ncu tp8 case ok", flush=True)


_OUR_KERNELS = ("gemm_kernel", "gemm_pair_kernel", "mix_units_kernel", "dequant_units_kernel",
                "gategrad_reduce_kernel", "loss_fused_kernel", "loss_stats_kernel", "loss_combine_kernel",
                "loss_grad_kernel", "rmsnorm_fwd_kernel", "rmsnorm_bwd_kernel", "rope_kernel", "swiglu_kernel",
                "route_prep_kernel", "q8_0_quantize_kernel")


def _count_our_launches(fn):
    """Kernels of libvoodoo_b200 launched by one call of fn (CUPTI via torch.profiler)."""
    import torch

    try:
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
        return sum(1 for n in names if any(k in n for k in _OUR_KERNELS))
    except Exception:  # profiler unavailable: no claim
        return None


def _print_step_profile(fn, top: int = 30):
    """Device time per kernel name over one call of fn (CUPTI via torch.profiler),
    printed to stderr as a table: name, launches, total ms, share."""
    import torch

    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    agg = {}
    for e in prof.events():
        if e.device_type != torch.autograd.DeviceType.CUDA:
            continue
        n, t = agg.get(e.name, (0, 0.0))
        agg[e.name] = (n + 1, t + e.device_time_total / 1e3)
    total = sum(t for _, t in agg.values()) or 1.0
    print(f"[step profile] {len(agg)} kernel names, {sum(n for n, _ in agg.values())} launches, "
          f"{total:.2f} ms device time", file=sys.stderr)
    for name, (n, t) in sorted(agg.items(), key=lambda kv: -kv[1][1])[:top]:
        print(f"[step profile] {t:9.3f} ms {100 * t / total:5.1f}% {n:6d}x  {name[:110]}", file=sys.stderr)


def step_flops_per_token(shape) -> float:
    """Algorithmic FLOPs per token of the distillation step: student linear
    layers 6 x params (forward, dX and the gate-gradient GEMM), a tied
    (unquantised) student head 4 x params (forward and dX), an untied gated
    head 6 x, the teacher 2 x its linear params, and causal attention
    4 * L * (S / 2) * d_attn per token forward (x3 student, x1 teacher)."""
    hd = shape.head_dim or shape.hidden // shape.heads
    d_attn = shape.heads * hd
    p_layers = shape.layers * (shape.hidden * (shape.heads + 2 * shape.kv_heads) * hd + d_attn * shape.hidden +
                               3 * shape.hidden * shape.ffn)
    p_head = shape.vocab * shape.hidden
    student = 6 * p_layers + (4 if shape.tied else 6) * p_head
    teacher = 2 * (p_layers + p_head)
    attn = 4 * shape.layers * (shape.seq / 2) * d_attn * 4
    return float(student + teacher + attn)


def auto_teacher_tp(workload: str, world: int) -> int:
    """The teacher's TP degree by default: the smallest t dividing the
    world whose world / t groups each get a whole number of the batch's
    sequences (each group runs the teacher on its slice, so fewer ranks
    share each teacher all-reduce, or none at t = 1); 0 (the student's
    degree) on one GPU or when none fits."""
    if world <= 1 or workload not in WORKLOAD_NAMES:
        return 0
    from voodoo_quant.training import synthetic as S

    batch = S.SHAPES[workload].batch
    for t in range(1, world + 1):
        if world % t == 0 and batch % (world // t) == 0:
            return t if t < world else 0
    return 0


def run_model_step(args):
    """Full gated distillation step of a synthetic model config: student
    (every Linear and the embedding gated, K candidates) forward, Q8_0 teacher
    forward, fused CE + T^2 KL loss, size term, backward, clip, AdamW and
    cosine LR.  Tokens per step = batch x seq.  Under torchrun (N > 1) both
    models are tensor-parallel over the N GPUs (Llama adapter: q/k/v by heads,
    o row-parallel, gate/up column, down row, vocab-parallel embedding, head
    and loss) and every rank runs the same batch; value = tokens / max-over-
    ranks step time."""
    import torch
    import torch.distributed as dist
    from voodoo_quant import _C
    from voodoo_quant.training import synthetic as S
    from voodoo_quant.training.trainer import StepArgs, build_distill

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        from voodoo_quant import parallel

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
        parallel.adopt_process_group(local)
    _C.load_library()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # the metric's second half (mix-GEMM kernels of config 2), on rank 0's GPU
    # before the model is built
    mix_gemm = layer_kernel_fractions(dev, args.kernel_iters) if rank == 0 and not args.no_layer_kernels else None

    workload = args.workload
    if args.layers > 0:
        # a smoke run of the workload's build, memory plan and step with fewer
        # decoder layers: a different (smaller) model, so its line names it
        import dataclasses

        base = S.SHAPES[args.workload]
        workload = f"{args.workload}-{args.layers}l"
        S.SHAPES[workload] = dataclasses.replace(base, layers=args.layers)
    t_build = time.perf_counter()
    trainer, shape = build_distill(workload, dev, seed=0, tp=world > 1,
                                   overlap_sms=args.overlap_sms if world > 1 else 0,
                                   args=StepArgs(max_steps=args.warmup + args.steps + args.e2e_steps + 3,
                                                 ptqr=args.ptqr, logits_chunk=args.logits_chunk,
                                                 ce_reduction="tokens" if args.logits_chunk > 0 or args.graph_step
                                                 else "valid", static_shapes=args.graph_step,
                                                 teacher_tp=args.teacher_tp,
                                                 joint_teacher=bool(args.joint_teacher),
                                                 joint_teacher_sms=args.joint_teacher_sms,
                                                 sequence_parallel=args.sequence_parallel and world > 1))
    torch.cuda.synchronize()
    t_build = time.perf_counter() - t_build
    x, y = S.random_tokens(shape, dev, seed=1)
    tokens = x.numel()
    stream = torch.cuda.current_stream()
    torch.cuda.reset_peak_memory_stats(dev)
    step_fn = trainer.step
    graph_note = "eager"
    if args.graph_step:  # forward + backward recorded once, replayed per step (optimizer eager)
        ok, err = 1.0, ""
        try:
            trainer.capture(x, y, warmup=args.warmup)
        except Exception as e:  # capture unsupported here: every rank falls back to the eager step
            ok, err = 0.0, f"{type(e).__name__}: {str(e)[:120]}"
            trainer.release_graph()
            torch.cuda.synchronize()
        flag = torch.tensor([ok], device=dev)
        if world > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if flag.item() == 1.0:
            step_fn = trainer.replay_step
            graph_note = "forward + backward replayed from one CUDA graph"
        else:
            trainer.release_graph()
            graph_note = f"eager (graph capture failed: {err or 'on another rank'})"
            if rank == 0:
                print(f"[bench] {graph_note}", file=sys.stderr, flush=True)
    for _ in range(args.warmup):
        step_fn(x, y)
    torch.cuda.synchronize()
    peak_gb = torch.cuda.max_memory_allocated(dev) / 1e9
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local).start()
    barrier()
    torch.cuda.synchronize()
    clk.mark_start()
    ev0.record(stream)
    for _ in range(args.steps):
        out = step_fn(x, y)
    ev1.record(stream)
    torch.cuda.synchronize()
    clk.mark_end()
    barrier()
    clk.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    assert torch.isfinite(out["loss"]).item() and _C.device_error() == 0

    # e2e: token ids from pinned host memory each step, the loss read back each step
    xh, yh = x.cpu().pin_memory(), y.cpu().pin_memory()
    lh = torch.empty((), dtype=torch.float32).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.e2e_steps):
        xd = xh.to(dev, non_blocking=True)
        yd = yh.to(dev, non_blocking=True)
        o = step_fn(xd, yd)
        lh.copy_(o["loss"], non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.e2e_steps)
    launches = _count_our_launches(lambda: step_fn(x, y))
    if args.profile_step:
        _print_step_profile(lambda: step_fn(x, y)) if rank == 0 else step_fn(x, y)
    if args.ncu_step:  # one more step inside cudaProfilerStart/Stop, for ncu --profile-from-start off
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        step_fn(x, y)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    torch.cuda.synchronize()

    if rank == 0:
        pk, pk_kind = peaks()
        peak_t = float(pk.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
        fpt = step_flops_per_token(shape)
        ach = fpt * tokens / (ms * 1e-3) / 1e12
        cfg = step_config(args.workload, shape, world)
        if args.layers > 0:
            cfg["workload"] += (f" -- SMOKE RUN with {shape.layers} of {S.SHAPES[args.workload].layers} layers, "
                                "not the configuration")
        res = {
            "metric": METRIC,
            "value": round(tokens / (ms * 1e-3), 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 3),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded random-init weights and tokens; candidates from the round-to-nearest packer)",
            "config": cfg,
            "run": {"gated_tensors": len(trainer.replaced), "build_s": round(t_build, 1),
                    "input_grad_overlap_sms": args.overlap_sms if world > 1 else 0,
                    "forward": "ptqr (one candidate per token)" if args.ptqr else "candidate mixture",
                    "logits_chunk": args.logits_chunk, "peak_alloc_gb_rank0": round(peak_gb, 2),
                    "step_graph": graph_note,
                    "teacher_tp": args.teacher_tp or world,
                    "teacher_batch_slices": world // (args.teacher_tp or world),
                    "sequence_parallel": bool(args.sequence_parallel and world > 1),
                    "teacher": (f"layers interleaved with the student's forward all-reduces, "
                                f"{args.joint_teacher_sms} SMs left to them") if trainer._joint_ok()
                    else "after the student, same stream"},
            "roofline": {"bound": "tensor", "kernel": "whole step (tcgen05 GEMMs dominate)", "flops_per_token": fpt,
                         "achieved": round(ach, 1), "peak": round(peak_t * world, 1), "unit": "TFLOP/s",
                         "frac": round(ach / (peak_t * world), 4),
                         "peak_source": f"{pk_kind} bf16_tflops_sustained x {world} GPUs", "traffic": None},
            "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(2 * tokens * 8), "d2h_bytes_per_step": 4},
            "gpu_launches": launches * args.steps if launches is not None else None,
            "clocks": clk.summary(),
            "loss_last": round(float(out["loss"]), 4),
            "size_bytes_last": float(out["size_bytes"]),
        }
        if mix_gemm is not None:
            res["mix_gemm"] = mix_gemm
        if world == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = step_cpu_baseline(shape, tokens=args.cpu_tokens)
        print(json.dumps(res), flush=True)
    trainer.release_graph()  # the graph holds collectives: drop it before the process group
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_cache_load(args):
    """Candidate-cache load (the store's I/O row): combined_lazy cache files
    holding the six packed candidates (Q2_K..Q8_0) of 8B MLP-shaped tensors
    [14336 x 4096] are memory-mapped and packed into HBM arenas, through the
    pinned double-buffered staging (``cache.upload_staged``) and, for
    comparison, through plain pageable copies.  Files are written first, so
    the page cache is warm: this measures the host->HBM path, not the disk."""
    import tempfile

    import torch
    from voodoo_quant import cache
    from voodoo_quant.cache import pack_arena
    from voodoo_quant.quants import rtn

    dev = torch.device("cuda", 0)
    types = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]
    rows, cols, n_files = 14336, 4096, 4
    with tempfile.TemporaryDirectory() as td:
        paths = []
        for i in range(n_files):
            g = torch.Generator(device=dev).manual_seed(i)
            w = torch.randn(rows, cols, device=dev, generator=g) * 0.02
            qb = {qt: rtn.quantize(w, qt).cpu() for qt in types}
            paths.append(os.path.join(td, f"combined_lazy_w{i:016x}_inone.pt"))
            torch.save(qb, paths[-1])
            del w, qb
        nbytes = 0

        def load_all():
            nonlocal nbytes
            nbytes = 0
            arenas = []
            for p in paths:
                mm = torch.load(p, weights_only=True, map_location="cpu", mmap=True)
                a, lay = pack_arena(types, [mm[qt] for qt in types], rows, cols, dev)
                nbytes += sum(l.nbytes for l in lay)
                arenas.append(a)
            torch.cuda.synchronize()
            return arenas

        res = {}
        for mode in ("staged", "pageable", "staged"):
            cache._STAGE_MIN = (1 << 20) if mode == "staged" else (1 << 62)
            t0 = time.perf_counter()
            arenas = load_all()
            dt = time.perf_counter() - t0
            res[mode] = nbytes / dt / 1e9
            del arenas
        cache._STAGE_MIN = 1 << 20
    print(json.dumps({"metric": "candidate cache load (mmap -> HBM arena)", "value": round(res["staged"], 2),
                      "unit": "GB/s", "n_gpus": 1, "higher_is_better": True,
                      "pageable_copy_gbs": round(res["pageable"], 2), "bytes_per_load": nbytes,
                      "config": {"workload": f"{n_files} combined_lazy files, 6 candidates of [{rows}x{cols}]",
                                 "page_cache": "warm", "staging": f"2 x {cache._STAGE_BYTES >> 20} MiB pinned"}}),
          flush=True)


def run_gemm_shapes(args):
    """The gated Linear's kernels at every distinct projection shape of the
    8B step (one GPU, T = 16384 tokens): per shape and TP degree (1 and 8:
    the rank's shard), the mixture, forward, dX and gate-gradient GEMMs timed
    with CUDA events (after 2 warm-up calls, ``--kernel-iters`` timed),
    as TFLOP/s (2 T N Kin each) and fractions of the measured burst peak;
    six candidates Q2_K..Q8_0.  Inputs are larger than L2 for the large
    shapes; small shards partly live in L2, as they do in the step."""
    import torch
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn
    from voodoo_quant.training import synthetic as S

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = S.SHAPES["8b"]
    types = list(shape.candidates)
    T = shape.batch * shape.seq
    pk, pk_kind = peaks()
    peak_t = float(pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    g = torch.Generator(device=dev).manual_seed(0)
    rows = []
    seen = set()
    for tp in (1, 8):
        for role, n_out, n_in, _ in layer_linear_shapes(shape) + [("lm_head", shape.vocab, shape.hidden, None)]:
            if role in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj", "lm_head"):
                n, kin = n_out // tp, n_in  # column-parallel: output rows split
            else:
                n, kin = n_out, n_in // tp  # row-parallel: input columns split
            key = (n, kin)
            if key in seen:
                continue
            seen.add(key)
            w = torch.randn(n, kin, device=dev, generator=g) * 0.02
            blocks = [rtn.quantize(w, q) for q in types]
            del w
            probs = torch.softmax(torch.randn(len(types), device=dev, generator=g), 0)
            x = torch.randn(T, kin, device=dev, generator=g).to(torch.bfloat16)
            dy = torch.randn(T, n, device=dev, generator=g).to(torch.bfloat16)
            wm = _C.mix(types, blocks, probs, n, kin, kin)
            ws = torch.empty(max(_C.gategrad_workspace_bytes(n, kin, len(types)), 4), dtype=torch.uint8, device=dev)
            fns = {"mix": lambda: _C.mix(types, blocks, probs, n, kin, kin, out=wm),
                   "fwd": lambda: _C.linear_fwd(x, wm, n, kin),
                   "dx": lambda: _C.linear_dx(dy, wm, kin),
                   "gategrad": lambda: _C.gategrad(dy, x, types, blocks, n, kin, kin, workspace=ws)}
            res = {"role": role, "tp": tp, "N": n, "Kin": kin}
            for name, fn in fns.items():
                for _ in range(2):
                    fn()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                fn()  # the timed launches queue behind this one, so host launch time stays hidden
                e0.record()
                for _ in range(args.kernel_iters):
                    fn()
                e1.record()
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / args.kernel_iters
                if name == "mix":
                    res["mix_ms"] = round(ms, 4)
                else:
                    tf = 2.0 * T * n * kin / (ms * 1e-3) / 1e12
                    res[name] = {"ms": round(ms, 4), "TFLOP/s": round(tf, 1), "frac": round(tf / peak_t, 3)}
            rows.append(res)
            del blocks, x, dy, wm, ws
            torch.cuda.empty_cache()
    assert _C.device_error() == 0
    print(json.dumps({"metric": "gated-Linear kernels per 8B projection shape", "tokens": T, "candidates": types,
                      "peak_tflops": peak_t, "peak_source": f"{pk_kind} bf16_tflops (burst)", "shapes": rows}),
          flush=True)


def _time_fn(fn, iters):
    """ms per call of fn with CUDA events (2 warm-up calls; the timed calls
    queue behind one more, so host launch time stays hidden)."""
    import torch

    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    fn()
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def run_fused_mix(args):
    """The forward of a gated Linear two ways (one GPU): the mix kernel
    writing W_mix to HBM and the GEMM reading it, against one GEMM whose
    producer warps decode and mix the operand tiles in shared memory
    (``vq_mixgemm_fwd_fused``).  Config 2 (K = 5) and the teacher's K = 1
    Q8_0 decode at two 8B projection shapes (T = 16384)."""
    import torch
    from voodoo_quant import _C
    from voodoo_quant.quants import rtn

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pk, pk_kind = peaks()
    peak_t = float(pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    g = torch.Generator(device=dev).manual_seed(0)
    cases = [("config2", T_TOK, 14336, 4096, list(TYPES)),
             ("teacher gate|up 8B", 16384, 28672, 4096, ["Q8_0"]),
             ("teacher down 8B", 16384, 4096, 14336, ["Q8_0"])]
    rows = []
    for name, T, n, kin, types in cases:
        w = torch.randn(n, kin, device=dev, generator=g) * 0.02
        blocks = [rtn.quantize(w, q) for q in types]
        del w
        probs = torch.softmax(torch.randn(len(types), device=dev, generator=g), 0)
        x = torch.randn(T, kin, device=dev, generator=g).to(torch.bfloat16)
        wm = _C.mix(types, blocks, probs, n, kin, kin)
        y = torch.empty(T, n, dtype=torch.bfloat16, device=dev)
        t_mix = _time_fn(lambda: _C.mix(types, blocks, probs, n, kin, kin, out=wm), args.kernel_iters)
        t_fwd = _time_fn(lambda: _C.linear_fwd(x, wm, n, kin, out=y), args.kernel_iters)
        t_fused = _time_fn(lambda: _C.mixgemm_fwd_fused(x, types, blocks, probs, n, kin, kin, out=y),
                           args.kernel_iters)
        tf = 2.0 * T * n * kin / 1e12
        rows.append({"case": name, "T": T, "N": n, "Kin": kin, "candidates": types, "mix_ms": round(t_mix, 4),
                     "gemm_ms": round(t_fwd, 4), "separate_ms": round(t_mix + t_fwd, 4),
                     "fused_ms": round(t_fused, 4), "fused_TFLOP/s": round(tf / (t_fused * 1e-3), 1),
                     "fused_frac": round(tf / (t_fused * 1e-3) / peak_t, 3)})
        del blocks, x, wm, y
        torch.cuda.empty_cache()
    assert _C.device_error() == 0
    print(json.dumps({"metric": "gated-Linear forward: mix + GEMM vs decoded-operand GEMM", "peak_tflops": peak_t,
                      "peak_source": f"{pk_kind} bf16_tflops (burst)", "cases": rows}), flush=True)


def run_collectives(args):
    """The TP group's collectives alone (torchrun, one process per GPU): NCCL
    all-reduce, reduce-scatter and all-gather of bf16 tensors the size of the
    8B step's hidden state ([16384, 4096] = 134.2 MB) and an eighth of it,
    after 5 warm-up calls, 20 calls timed with CUDA events, max over ranks.
    Bus bandwidth in the nccl-tests convention (all-reduce 2 (N - 1) / N,
    reduce-scatter and all-gather (N - 1) / N of the full tensor's bytes)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2:
        print(json.dumps({"metric": "collectives", "unavailable": "needs torchrun with 2 or more GPUs"}))
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    res = {}
    for mb in (16.8, 134.2):
        n = int(mb * 1e6 / 2)
        n -= n % (world * 8)
        x = torch.randn(n, device=dev).to(torch.bfloat16)
        shard = torch.empty(n // world, device=dev, dtype=torch.bfloat16)
        full = torch.empty(n, device=dev, dtype=torch.bfloat16)
        for op in ("all_reduce", "reduce_scatter", "all_gather"):
            def f():
                if op == "all_reduce":
                    dist.all_reduce(x)
                elif op == "reduce_scatter":
                    dist.reduce_scatter_tensor(shard, x)
                else:
                    dist.all_gather_into_tensor(full, shard)
            for _ in range(5):
                f()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(20):
                f()
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) / 20], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            factor = 2 * (world - 1) / world if op == "all_reduce" else (world - 1) / world
            res[f"{op}_{mb}MB"] = {"ms": round(ms, 4), "bus_GBps": round(n * 2 * factor / (ms * 1e-3) / 1e9, 1)}
    if rank == 0:
        print(json.dumps({"metric": "TP collectives (bf16)", "n_gpus": world, "results": res,
                          "nccl": ".".join(str(v) for v in torch.cuda.nccl.version())}), flush=True)
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", choices=["8b", "layer", "tiny", "0.6b", "32b", "cache-load", "collectives",
                                           "gemm-shapes", "fused-mix"],
                    default="8b",
                    help="8b (default): the config-4 distillation step at TP-N; tiny/0.6b/32b: the other step "
                         "configurations (32b: the TP-4 / TP-8 case, K=7 with per-role menus); layer: the config-2 "
                         "single gated-Linear step; cache-load: candidate-cache files into HBM (GB/s); "
                         "collectives: the TP group's NCCL all-reduce / reduce-scatter / all-gather alone; "
                         "gemm-shapes: the gated Linear's kernels at every 8B projection shape (TP-1 and TP-8 shards); "
                         "fused-mix: the forward as mix + GEMM against one GEMM decoding its operand tiles")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--kernel-iters", type=int, default=10)
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-tokens", type=int, default=-1,
                    help="host sample tokens (default: 256 for step workloads, 2048 for the layer)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-layer-kernels", action="store_true",
                    help="step workloads: skip the config-2 mix-GEMM kernel fractions (mix_gemm key)")
    ap.add_argument("--no-graph", action="store_true", help="layer workload: time the eager step, not a CUDA graph")
    ap.add_argument("--overlap-sms", type=int, default=-1,
                    help="TP: SMs the gate-gradient GEMMs leave to the concurrent input-gradient all-reduces, which "
                         "run on a communicator capped to that many CTAs (default: 32 with more than one GPU, "
                         "0 otherwise)")
    ap.add_argument("--dx-chunks", type=int, default=-1,
                    help="layer workload under TP: row chunks of dX, each all-reduced while the next is computed "
                         "(default: 2 with more than one GPU)")
    ap.add_argument("--ptqr", action="store_true",
                    help="step workloads: per-token quant routing forward (one candidate per token)")
    ap.add_argument("--logits-chunk", type=int, default=0,
                    help="step workloads: head + loss per chunk of this many tokens (no [tokens, V] logits)")
    ap.add_argument("--graph-step", action=argparse.BooleanOptionalAction, default=None,
                    help="step workloads: record forward + backward as one CUDA graph (static-shape mode, "
                         "CE over all tokens) and replay it each step; the optimizer stays eager "
                         "(default: on with more than one GPU)")
    ap.add_argument("--teacher-tp", type=int, default=-1,
                    help="step workloads under TP: the teacher's own TP degree t (groups of t ranks, each on "
                         "its batch slice; one all-to-all of its logits); 0 = the student's; default: the "
                         "smallest t whose groups split the batch evenly")
    ap.add_argument("--joint-teacher", action=argparse.BooleanOptionalAction, default=None,
                    help="step workloads under TP with a TP-1 teacher on each rank's batch slice: issue each "
                         "teacher decoder block while the matching student block's forward all-reduce is in flight "
                         "(default: on with 4 or more GPUs, where it was measured faster)")
    ap.add_argument("--joint-teacher-sms", type=int, default=32,
                    help="with --joint-teacher: SMs the teacher's GEMMs leave to the all-reduce in flight")
    ap.add_argument("--sequence-parallel", action=argparse.BooleanOptionalAction, default=False,
                    help="step workloads under TP: residual stream, norms and residual adds on token shards; "
                         "all-gather / reduce-scatter around each block instead of all-reduces")
    ap.add_argument("--layers", type=int, default=0,
                    help="step workloads: build only this many decoder layers (a smoke run of the build, "
                         "memory plan and step; its line says so and is not the configuration's number)")
    ap.add_argument("--ncu-step", action="store_true",
                    help="step workloads: after the timed region, run one more step between cudaProfilerStart and "
                         "cudaProfilerStop (for ncu --profile-from-start off: that step's launches only)")
    ap.add_argument("--profile-step", action="store_true",
                    help="step workloads: print device time per kernel name for one step")
    ap.add_argument("--ncu-case", nargs="?", const="config2", default=None, choices=["config2", "tp8"],
                    help="one launch per kernel at profiling sizes (config2: mix, GEMMs, loss; tp8: the GEMMs at two "
                         "TP-8 shard shapes)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.overlap_sms < 0:
        # NCCL's default channel count here: at TP-2 it measured 1.262 ms per
        # layer step against 1.286 ms with 24 (and 1.30 ms without overlap);
        # with more ranks the all-reduce outlasts the gate-gradient GEMM
        args.overlap_sms = 32 if world > 1 else 0
    if args.dx_chunks < 0:
        args.dx_chunks = 2 if world > 1 else 1
    if args.cpu_tokens < 0:
        args.cpu_tokens = 2048 if args.workload == "layer" else 256
    if args.graph_step is None:
        args.graph_step = world > 1 and args.workload != "layer" and args.logits_chunk <= 0 and not args.ptqr
    if args.teacher_tp < 0:
        args.teacher_tp = auto_teacher_tp(args.workload, world) if args.logits_chunk <= 0 else 0
    if args.joint_teacher is None:
        args.joint_teacher = world >= 4
    if args.ncu_case == "tp8":
        run_ncu_case_tp8()
    elif args.ncu_case:
        run_ncu_case()
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "cache-load":
        run_cache_load(args)
    elif args.workload == "collectives":
        run_collectives(args)
    elif args.workload == "gemm-shapes":
        run_gemm_shapes(args)
    elif args.workload == "fused-mix":
        run_fused_mix(args)
    elif args.workload != "layer":
        run_model_step(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
