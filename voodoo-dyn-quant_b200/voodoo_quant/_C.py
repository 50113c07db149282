"""ctypes binding of libvoodoo_b200.so (the sm_100a kernels) for torch tensors.

The library is loaded from this package directory (built in-tree by
``__graft_entry__.build()``).  There is no fallback: if the library is
missing, or CUDA is not available, every entry point raises ``RuntimeError``.
Status codes of the C ABI map onto the reference's exception conventions:
invalid shapes / alignment / unknown quant types raise ``ValueError``
(voodoo_quant/ggml.py:161-164,195-198,242-253 in the reference), CUDA
failures raise ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_NAME = "libvoodoo_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

VQ_ERR_INVALID = -1
VQ_ERR_CUDA = -2
VQ_ERR_UNSUPPORTED = -3

# ggml type ids of the supported candidate formats.
GGML_TYPE = {"Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ4_XS": 23}

_lib = None

_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_int = ctypes.c_int
_f32 = ctypes.c_float


def _declare(lib):
    sig = {
        "vq_last_error": (ctypes.c_char_p, []),
        "vq_abi_version": (_int, []),
        "vq_format_info": (_int, [_int, ctypes.POINTER(_int), ctypes.POINTER(_int)]),
        "vq_device_error": (_int, [_vp, ctypes.POINTER(_int)]),
        "vq_dequant": (_int, [_int, _vp, _i64, _i64, _vp, _vp]),
        "vq_quantize": (_int, [_int, _vp, _int, _i64, _i64, _i64, _vp, _vp]),
        "vq_mix": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp]),
        "vq_linear_fwd": (_int, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp]),
        "vq_linear_fwd_swiglu": (_int, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp]),
        "vq_set_gategrad_sm_reserve": (_int, [_int]),
        "vq_set_gemm_sm_reserve": (_int, [_int]),
        "vq_route_prep": (_int, [_vp, _i64, _int, _vp, _vp, _vp, _vp]),
        "vq_linear_fwd_grouped": (_int, [_vp, _i64, _i64, _i64, _int, _vp, _i64, _i64, _vp, _vp, _i64, _vp]),
        "vq_linear_dx": (_int, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp]),
        "vq_gategrad_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _int]),
        "vq_gategrad": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _int, _vp, _vp, _i64, _vp,
                               ctypes.c_size_t, _vp, _vp]),
        "vq_gategrad_noalloc": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _int, _vp, _vp, _i64, _vp, _vp]),
        "vq_gategrad_grouped_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _int, _int]),
        "vq_gategrad_grouped": (_int, [_vp, _i64, _vp, _i64, _i64, _int, _vp, _i64, _int, _vp, _vp, _i64, _vp,
                                       ctypes.c_size_t, _vp, _i64, _vp]),
        "vq_mixgemm_fwd": (_int, [_vp, _i64, _i64, _i64, _int, _vp, _vp, _vp, _i64, _i64, _vp, _i64, _vp,
                                  _i64, _vp]),
        "vq_mixgemm_fwd_fused": (_int, [_vp, _i64, _i64, _i64, _int, _vp, _vp, _vp, _i64, _i64, _vp, _i64,
                                        _vp]),
        "vq_mixgemm_dx": (_int, [_vp, _i64, _i64, _i64, _int, _vp, _vp, _vp, _i64, _i64, _vp, _i64, _vp,
                                 _i64, _vp]),
        "vq_loss_fused": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _f32, _f32, _f32, _vp, _vp, _vp,
                                 _i64, _vp]),
        "vq_loss_stats": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _f32, _vp, _vp]),
        "vq_loss_combine": (_int, [_vp, _int, _i64, _f32, _vp, _vp, _vp, _vp]),
        "vq_loss_grad": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _f32, _vp, _f32, _f32, _vp,
                                _i64, _vp]),
        "vq_rmsnorm_fwd": (_int, [_vp, _i64, _i64, _i64, _vp, _f32, _vp, _i64, _vp, _vp]),
        "vq_rmsnorm_bwd": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _vp]),
        "vq_add_rmsnorm_fwd": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _f32, _vp, _i64, _vp, _i64, _vp, _vp]),
        "vq_rmsnorm_bwd_add": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _vp]),
        "vq_rope": (_int, [_vp, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _vp, _vp]),
        "vq_swiglu_fwd": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp]),
        "vq_swiglu_bwd": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return sig.keys()


EXPORTED = (
    "vq_last_error", "vq_abi_version", "vq_format_info", "vq_device_error", "vq_dequant", "vq_mix",
    "vq_linear_fwd", "vq_linear_fwd_swiglu", "vq_linear_fwd_grouped", "vq_set_gategrad_sm_reserve", "vq_set_gemm_sm_reserve", "vq_quantize", "vq_route_prep", "vq_linear_dx", "vq_gategrad_workspace_bytes", "vq_gategrad", "vq_gategrad_noalloc",
    "vq_gategrad_grouped_workspace_bytes", "vq_gategrad_grouped",
    "vq_mixgemm_fwd", "vq_mixgemm_fwd_fused", "vq_mixgemm_dx",
    "vq_loss_fused", "vq_loss_stats", "vq_loss_combine", "vq_loss_grad",
    "vq_rmsnorm_fwd", "vq_rmsnorm_bwd", "vq_add_rmsnorm_fwd", "vq_rmsnorm_bwd_add", "vq_rope", "vq_swiglu_fwd", "vq_swiglu_bwd",
)


def load_library(path: str | os.PathLike | None = None):
    """Load (once) and return the ctypes handle; raises RuntimeError if absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{LIB_NAME} not found at {p}; build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(the B200 path has no CPU fallback)"
        )
    lib = ctypes.CDLL(str(p))
    _declare(lib)
    if path is None:
        _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc == 0:
        return
    msg = _lib.vq_last_error().decode(errors="replace")
    if rc in (VQ_ERR_INVALID, VQ_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(f"libvoodoo_b200: {msg}")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(*ts: torch.Tensor) -> None:
    load_library()
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("libvoodoo_b200 kernels need CUDA tensors (no CPU fallback)")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def format_info(qtype: str) -> tuple[int, int]:
    lib = load_library()
    be, bb = _int(), _int()
    rc = lib.vq_format_info(GGML_TYPE.get(qtype, -1), ctypes.byref(be), ctypes.byref(bb))
    _check(rc)
    return be.value, bb.value


def device_error(device: torch.device | None = None) -> int:
    """Synchronise the current stream and return/clear the device error word."""
    lib = load_library()
    code = _int()
    st = torch.cuda.current_stream(device).cuda_stream
    _check(lib.vq_device_error(st, ctypes.byref(code)))
    return code.value


def quantize(w: torch.Tensor, qtype: str) -> torch.Tensor:
    """GPU quantiser: float32 / bfloat16 [rows, cols] -> uint8 [rows * cols / 32, 34] Q8_0 blocks
    (byte-identical to ggml's reference rule); other types raise ValueError."""
    _require_cuda(w)
    if qtype not in GGML_TYPE:
        raise ValueError(f"Unknown quant type: {qtype}. Supported: {list(GGML_TYPE)}")
    if w.dim() != 2:
        raise ValueError(f"quantize expects a 2-D weight, got shape {tuple(w.shape)}")
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.to(torch.float32)
    if w.stride(1) != 1:
        w = w.contiguous()
    be, bb = format_info(qtype)
    rows, cols = w.shape
    out = torch.empty(rows * (cols // be) if cols % be == 0 else 0, bb, dtype=torch.uint8, device=w.device)
    _check(_lib.vq_quantize(GGML_TYPE[qtype], w.data_ptr(), 0 if w.dtype == torch.float32 else 1, rows, cols,
                            w.stride(0), out.data_ptr(), _stream(w)))
    return out


def dequant(qbytes: torch.Tensor, qtype: str, rows: int, cols: int) -> torch.Tensor:
    """Bit-exact decode of packed blocks -> float32 [rows, cols] on the blocks' device."""
    _require_cuda(qbytes)
    if qtype not in GGML_TYPE:
        raise ValueError(f"Unknown quant type: {qtype}. Supported: {list(GGML_TYPE)}")
    be, bb = format_info(qtype)
    if cols % be:
        raise ValueError(f"{qtype} requires in_features % {be} == 0, got {cols}")
    if qbytes.numel() != rows * (cols // be) * bb:
        raise ValueError(
            f"qweight size {qbytes.numel()} does not match {rows * (cols // be)} blocks of {bb} bytes for {qtype}"
        )
    qb = qbytes.contiguous()
    out = torch.empty(rows, cols, dtype=torch.float32, device=qb.device)
    _check(_lib.vq_dequant(GGML_TYPE[qtype], qb.data_ptr(), rows, cols, out.data_ptr(), _stream(qb)))
    return out


def _cand_arrays(qtypes, qbytes):
    K = len(qtypes)
    types = (_int * K)(*[GGML_TYPE[q] for q in qtypes])
    ptrs = (_vp * K)(*[q.data_ptr() for q in qbytes])
    return K, types, ptrs


def mix(qtypes, qbytes, probs: torch.Tensor, rows: int, padded_cols: int, cols: int,
        out: torch.Tensor | None = None) -> torch.Tensor:
    """W_mix = sum_k probs[k] W_k -> bf16 [rows, ld] with ld = cols rounded up to 8."""
    _require_cuda(probs, *qbytes)
    ld = (cols + 7) // 8 * 8
    if out is None:
        out = torch.empty(rows, ld, dtype=torch.bfloat16, device=probs.device)
    K, types, ptrs = _cand_arrays(qtypes, qbytes)
    p = probs.detach().to(torch.float32).contiguous()
    _check(_lib.vq_mix(K, types, ptrs, p.data_ptr(), rows, padded_cols, cols, out.data_ptr(), out.stride(0),
                       _stream(p)))
    return out


def _as_operand(x: torch.Tensor) -> torch.Tensor:
    """bf16, unit column stride, leading dimension a multiple of 8, 16B-aligned base."""
    x = x.to(torch.bfloat16)
    if x.stride(-1) != 1 or x.stride(0) % 8 != 0 or x.data_ptr() % 16 != 0:
        cols = x.shape[1]
        ld = (cols + 7) // 8 * 8
        buf = torch.zeros(x.shape[0], ld, dtype=torch.bfloat16, device=x.device)
        buf[:, :cols] = x
        return buf
    return x


def linear_fwd(x: torch.Tensor, w: torch.Tensor, n_out: int | None = None, in_features: int | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """y[T, N] = x[T, Kin] w[N, Kin]^T in bf16 with fp32 accumulation."""
    _require_cuda(x, w)
    kin = x.shape[1] if in_features is None else in_features
    N = w.shape[0] if n_out is None else n_out
    x = _as_operand(x)
    if out is None:
        out = torch.empty(x.shape[0], N, dtype=torch.bfloat16, device=x.device)
    _check(_lib.vq_linear_fwd(x.data_ptr(), x.shape[0], kin, x.stride(0), w.data_ptr(), N, w.stride(0),
                              out.data_ptr(), out.stride(0), _stream(x)))
    return out


def mixgemm_fwd_fused(x: torch.Tensor, qtypes, qbytes, probs: torch.Tensor, n_out: int, padded_cols: int,
                      in_features: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x W_mix^T with the mixture decoded into the GEMM's operand tiles
    (vq_mixgemm_fwd_fused); equal to ``mix`` then ``linear_fwd``."""
    _require_cuda(x, probs, *qbytes)
    kin = x.shape[1] if in_features is None else in_features
    x = _as_operand(x)
    K, types, ptrs = _cand_arrays(qtypes, qbytes)
    p = probs.to(torch.float32).contiguous()
    if out is None:
        out = torch.empty(x.shape[0], n_out, dtype=torch.bfloat16, device=x.device)
    _check(_lib.vq_mixgemm_fwd_fused(x.data_ptr(), x.shape[0], kin, x.stride(0), K, types, ptrs, p.data_ptr(), n_out,
                                     padded_cols, out.data_ptr(), out.stride(0), _stream(x)))
    return out


def linear_fwd_swiglu(x: torch.Tensor, w: torch.Tensor, F: int, in_features: int | None = None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """h[T, F] = silu(x w[:F]^T) * (x w[F:2F]^T) in one GEMM (gate|up rounded
    to bf16 before the activation); T > 128 and F a multiple of 128."""
    _require_cuda(x, w)
    kin = x.shape[1] if in_features is None else in_features
    x = _as_operand(x)
    if out is None:
        out = torch.empty(x.shape[0], F, dtype=torch.bfloat16, device=x.device)
    _check(_lib.vq_linear_fwd_swiglu(x.data_ptr(), x.shape[0], kin, x.stride(0), w.data_ptr(), F, w.stride(0),
                                     out.data_ptr(), out.stride(0), _stream(x)))
    return out


def linear_fwd_grouped(x: torch.Tensor, ws: list, n_out: int, in_features: int, group_off: torch.Tensor,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """y[rows of group g] = x[rows of group g] ws[g]^T; group_off (int32, device, G + 1) need not be on the host."""
    _require_cuda(x, *ws)
    x = _as_operand(x)
    G = len(ws)
    ptrs = (_vp * G)(*[w.data_ptr() for w in ws])
    if out is None:
        out = torch.empty(x.shape[0], n_out, dtype=torch.bfloat16, device=x.device)
    go = group_off.to(torch.int32).contiguous()
    _check(_lib.vq_linear_fwd_grouped(x.data_ptr(), x.shape[0], in_features, x.stride(0), G, ptrs, n_out,
                                      ws[0].stride(0), go.data_ptr(), out.data_ptr(), out.stride(0), _stream(x)))
    return out


def linear_dx(dy: torch.Tensor, w: torch.Tensor, in_features: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """dx[T, Kin] = dy[T, N] w[N, Kin]."""
    _require_cuda(dy, w)
    dy = _as_operand(dy)
    N = w.shape[0]
    if out is None:
        out = torch.empty(dy.shape[0], in_features, dtype=torch.bfloat16, device=dy.device)
    _check(_lib.vq_linear_dx(dy.data_ptr(), dy.shape[0], N, dy.stride(0), w.data_ptr(), in_features, w.stride(0),
                             out.data_ptr(), out.stride(0), _stream(dy)))
    return out


def route_prep(keys: torch.Tensor, K: int):
    """(order int64 [T], inv int64 [T], group_off int32 [K + 1]) of the stable grouping of uint8 keys."""
    _require_cuda(keys)
    keys = keys.to(torch.uint8).contiguous().reshape(-1)
    T = keys.numel()
    order = torch.empty(T, dtype=torch.int64, device=keys.device)
    inv = torch.empty(T, dtype=torch.int64, device=keys.device)
    off = torch.empty(K + 1, dtype=torch.int32, device=keys.device)
    _check(_lib.vq_route_prep(keys.data_ptr(), T, K, order.data_ptr(), inv.data_ptr(), off.data_ptr(), _stream(keys)))
    return order, inv, off


def set_gategrad_sm_reserve(sms: int) -> None:
    """SMs later gate-gradient GEMMs leave free for a concurrent collective (0 = none)."""
    _check(load_library().vq_set_gategrad_sm_reserve(int(sms)))


def set_gemm_sm_reserve(sms: int) -> None:
    """SMs later forward / dX GEMMs leave free for a concurrent collective (0 = none)."""
    _check(load_library().vq_set_gemm_sm_reserve(int(sms)))


def gategrad(dy: torch.Tensor, x: torch.Tensor, qtypes, qbytes, n_out: int, in_features: int, padded_cols: int,
             workspace: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """grad_probs[k] = <dy^T x, W_k> (float32 [K], into `out` when given); dW is never materialised."""
    _require_cuda(dy, x, *qbytes)
    dy = _as_operand(dy)
    x = _as_operand(x)
    K, types, ptrs = _cand_arrays(qtypes, qbytes)
    need = _lib.vq_gategrad_workspace_bytes(n_out, in_features, K)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 4), dtype=torch.uint8, device=x.device)
    if out is None:
        g = torch.empty(K, dtype=torch.float32, device=x.device)
    else:
        if out.dtype != torch.float32 or out.numel() != K or not out.is_contiguous():
            raise ValueError("gategrad: out must be a contiguous float32 tensor of K elements")
        g = out
    _check(_lib.vq_gategrad(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), x.shape[0], n_out, in_features,
                            K, types, ptrs, padded_cols, workspace.data_ptr(), workspace.numel(), g.data_ptr(),
                            _stream(x)))
    return g


def gategrad_noalloc(dy: torch.Tensor, x: torch.Tensor, qtypes, qbytes, n_out: int, in_features: int,
                     padded_cols: int) -> torch.Tensor:
    """``gategrad`` on the library's own fixed scratch (vq_gategrad_noalloc), for
    callers that cannot allocate device scratch; the result still needs a [K]
    output tensor.  Calls that overlap on the GPU race on the shared scratch."""
    _require_cuda(dy, x, *qbytes)
    dy = _as_operand(dy)
    x = _as_operand(x)
    K, types, ptrs = _cand_arrays(qtypes, qbytes)
    g = torch.empty(K, dtype=torch.float32, device=x.device)
    _check(_lib.vq_gategrad_noalloc(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), x.shape[0], n_out,
                                    in_features, K, types, ptrs, padded_cols, g.data_ptr(), _stream(x)))
    return g


def gategrad_workspace_bytes(n_out: int, in_features: int, K: int) -> int:
    return int(load_library().vq_gategrad_workspace_bytes(n_out, in_features, K))


def gategrad_grouped_workspace_bytes(n_total: int, in_features: int, G: int, K: int) -> int:
    return int(load_library().vq_gategrad_grouped_workspace_bytes(n_total, in_features, G, K))


def gategrad_grouped(dy: torch.Tensor, x: torch.Tensor, qtypes, qbytes_per_layer, rows, in_features: int,
                     padded_cols: int, workspace: torch.Tensor | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """grad[g, k] = <dy_g^T x, W_{g,k}> for layers g side by side in dy's
    columns (rows[g] each, a multiple of 32), all with the formats `qtypes`:
    one gate-gradient GEMM (float32 [G, K], into `out` -- rows K floats
    apart or further, unit column stride -- when given)."""
    G = len(rows)
    _require_cuda(dy, x, *[b for bs in qbytes_per_layer for b in bs])
    dy = _as_operand(dy)
    x = _as_operand(x)
    K = len(qtypes)
    types = (_int * K)(*[GGML_TYPE[q] for q in qtypes])
    ptrs = (_vp * (G * K))(*[b.data_ptr() for bs in qbytes_per_layer for b in bs])
    rws = (ctypes.c_int64 * G)(*[int(r) for r in rows])
    need = _lib.vq_gategrad_grouped_workspace_bytes(sum(rows), in_features, G, K)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 4), dtype=torch.uint8, device=x.device)
    if out is None:
        out = torch.empty(G, K, dtype=torch.float32, device=x.device)
    elif out.dtype != torch.float32 or out.dim() != 2 or tuple(out.shape) != (G, K) or out.stride(1) != 1:
        raise ValueError("gategrad_grouped: out must be float32 [G, K] with unit column stride")
    _check(_lib.vq_gategrad_grouped(dy.data_ptr(), dy.stride(0), x.data_ptr(), x.stride(0), x.shape[0], G, rws,
                                    in_features, K, types, ptrs, padded_cols, workspace.data_ptr(), workspace.numel(),
                                    out.data_ptr(), out.stride(0), _stream(x)))
    return out


def loss_fused(s: torch.Tensor, t: torch.Tensor, targets: torch.Tensor, temperature: float, ce_weight: float,
               kl_weight: float, want_grad: bool = True):
    """Row CE, row T^2*KL and (optionally) d/ds for bf16 logits [rows, V]."""
    _require_cuda(s, t, targets)
    s = s.to(torch.bfloat16)
    t = t.to(torch.bfloat16)
    if s.stride(-1) != 1:
        s = s.contiguous()
    if t.stride(-1) != 1:
        t = t.contiguous()
    y = targets.to(torch.int64).contiguous()
    rows, V = s.shape
    ce = torch.empty(rows, dtype=torch.float32, device=s.device)
    kl = torch.empty(rows, dtype=torch.float32, device=s.device)
    g = torch.empty(rows, V, dtype=torch.bfloat16, device=s.device) if want_grad else None
    _check(_lib.vq_loss_fused(s.data_ptr(), s.stride(0), t.data_ptr(), t.stride(0), y.data_ptr(), rows, V,
                              float(temperature), float(ce_weight), float(kl_weight), ce.data_ptr(), kl.data_ptr(),
                              _ptr(g), g.stride(0) if g is not None else V, _stream(s)))
    return ce, kl, g


def loss_stats(s: torch.Tensor, t: torch.Tensor, targets: torch.Tensor, vocab_start: int, temperature: float):
    _require_cuda(s, t, targets)
    s = s.to(torch.bfloat16)
    t = t.to(torch.bfloat16)
    y = targets.to(torch.int64).contiguous()
    rows, V = s.shape
    st = torch.empty(rows, 8, dtype=torch.float32, device=s.device)
    _check(_lib.vq_loss_stats(s.data_ptr(), s.stride(0), t.data_ptr(), t.stride(0), y.data_ptr(), vocab_start, rows,
                              V, float(temperature), st.data_ptr(), _stream(s)))
    return st


def loss_combine(stats: torch.Tensor, temperature: float):
    """stats [R, rows, 8] -> (row_lse [rows, 4], row_ce [rows], row_kl [rows])."""
    _require_cuda(stats)
    stats = stats.to(torch.float32).contiguous()
    R, rows = stats.shape[0], stats.shape[1]
    lse = torch.empty(rows, 4, dtype=torch.float32, device=stats.device)
    ce = torch.empty(rows, dtype=torch.float32, device=stats.device)
    kl = torch.empty(rows, dtype=torch.float32, device=stats.device)
    _check(_lib.vq_loss_combine(stats.data_ptr(), R, rows, float(temperature), lse.data_ptr(), ce.data_ptr(),
                                kl.data_ptr(), _stream(stats)))
    return lse, ce, kl


def loss_grad(s: torch.Tensor, t: torch.Tensor, targets: torch.Tensor, vocab_start: int, temperature: float,
              row_lse: torch.Tensor, ce_weight: float, kl_weight: float) -> torch.Tensor:
    _require_cuda(s, t, targets, row_lse)
    s = s.to(torch.bfloat16)
    t = t.to(torch.bfloat16)
    y = targets.to(torch.int64).contiguous()
    rows, V = s.shape
    g = torch.empty(rows, V, dtype=torch.bfloat16, device=s.device)
    _check(_lib.vq_loss_grad(s.data_ptr(), s.stride(0), t.data_ptr(), t.stride(0), y.data_ptr(), vocab_start, rows,
                             V, float(temperature), row_lse.contiguous().data_ptr(), float(ce_weight),
                             float(kl_weight), g.data_ptr(), g.stride(0), _stream(s)))
    return g


# ---------------------------------------------------------------- Llama block elementwise
def _rows_operand(t: torch.Tensor) -> torch.Tensor:
    """bf16 2-D view with unit column stride, 16-byte aligned rows."""
    t = t.to(torch.bfloat16)
    if t.stride(-1) != 1 or t.stride(0) % 8 != 0 or t.data_ptr() % 16 != 0:
        t = t.contiguous()
    return t


def rmsnorm_fwd(x: torch.Tensor, weight: torch.Tensor, eps: float):
    """(y [rows, D] bf16, rstd [rows] float32) for x [rows, D]."""
    _require_cuda(x, weight)
    x = _rows_operand(x)
    w = weight.to(torch.bfloat16).contiguous()
    rows, D = x.shape
    y = torch.empty(rows, D, dtype=torch.bfloat16, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    _check(_lib.vq_rmsnorm_fwd(x.data_ptr(), x.stride(0), rows, D, w.data_ptr(), float(eps), y.data_ptr(), y.stride(0),
                               rstd.data_ptr(), _stream(x)))
    return y, rstd


def rmsnorm_bwd(x: torch.Tensor, dy: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor) -> torch.Tensor:
    _require_cuda(x, dy, weight, rstd)
    x = _rows_operand(x)
    dy = _rows_operand(dy)
    w = weight.to(torch.bfloat16).contiguous()
    rows, D = x.shape
    dx = torch.empty(rows, D, dtype=torch.bfloat16, device=x.device)
    _check(_lib.vq_rmsnorm_bwd(x.data_ptr(), x.stride(0), dy.data_ptr(), dy.stride(0), rows, D, w.data_ptr(),
                               rstd.contiguous().data_ptr(), dx.data_ptr(), dx.stride(0), _stream(x)))
    return dx


def add_rmsnorm_fwd(a: torch.Tensor, res: torch.Tensor, weight: torch.Tensor, eps: float):
    """(h = a + res, y = RMSNorm(h), rstd) for a, res [rows, D] bf16."""
    _require_cuda(a, res, weight)
    a = _rows_operand(a)
    res = _rows_operand(res)
    w = weight.to(torch.bfloat16).contiguous()
    rows, D = a.shape
    if res.shape != a.shape:
        raise ValueError(f"add_rmsnorm: shapes {tuple(a.shape)} and {tuple(res.shape)} differ")
    h = torch.empty(rows, D, dtype=torch.bfloat16, device=a.device)
    y = torch.empty(rows, D, dtype=torch.bfloat16, device=a.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=a.device)
    _check(_lib.vq_add_rmsnorm_fwd(a.data_ptr(), a.stride(0), res.data_ptr(), res.stride(0), rows, D, w.data_ptr(),
                                   float(eps), h.data_ptr(), h.stride(0), y.data_ptr(), y.stride(0), rstd.data_ptr(),
                                   _stream(a)))
    return h, y, rstd


def rmsnorm_bwd_add(x: torch.Tensor, dy: torch.Tensor, dres: torch.Tensor, weight: torch.Tensor,
                    rstd: torch.Tensor) -> torch.Tensor:
    """RMSNorm input gradient of dy at x, plus dres (fp32 sum, one rounding)."""
    _require_cuda(x, dy, dres, weight, rstd)
    x = _rows_operand(x)
    dy = _rows_operand(dy)
    dres = _rows_operand(dres)
    w = weight.to(torch.bfloat16).contiguous()
    rows, D = x.shape
    dx = torch.empty(rows, D, dtype=torch.bfloat16, device=x.device)
    _check(_lib.vq_rmsnorm_bwd_add(x.data_ptr(), x.stride(0), dy.data_ptr(), dy.stride(0), dres.data_ptr(),
                                   dres.stride(0), rows, D, w.data_ptr(), rstd.contiguous().data_ptr(), dx.data_ptr(),
                                   dx.stride(0), _stream(x)))
    return dx


def _bshd(t: torch.Tensor) -> torch.Tensor:
    t = t.to(torch.bfloat16)
    if t.stride(-1) != 1 or any(st % 8 for st in t.stride()[:3]) or t.data_ptr() % 16 != 0:
        t = t.contiguous()
    return t


def rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, backward: bool = False):
    """Rotary embedding of q [B, S, Hq, D] and k [B, S, Hk, D] with cos/sin
    [B, S, D] (any strides with unit stride over D); returns contiguous
    [B, S, H, D] outputs (the transposed rotation when ``backward``)."""
    _require_cuda(q, k, cos, sin)
    q, k = _bshd(q), _bshd(k)
    B, S, Hq, D = q.shape
    Hk = k.shape[2]
    cos = cos.to(torch.bfloat16).expand(B, S, D)
    sin = sin.to(torch.bfloat16).expand(B, S, D)
    if cos.stride() != sin.stride() or cos.stride(-1) != 1 or cos.data_ptr() % 16 or sin.data_ptr() % 16 or \
            any(st % 8 for st in cos.stride()[:2]):
        cos, sin = cos.contiguous(), sin.contiguous()
    qo = torch.empty(B, S, Hq, D, dtype=torch.bfloat16, device=q.device)
    ko = torch.empty(B, S, Hk, D, dtype=torch.bfloat16, device=q.device)
    qs = (ctypes.c_int64 * 3)(q.stride(0), q.stride(1), q.stride(2))
    ks = (ctypes.c_int64 * 3)(k.stride(0), k.stride(1), k.stride(2))
    cs = (ctypes.c_int64 * 2)(cos.stride(0), cos.stride(1))
    _check(_lib.vq_rope(q.data_ptr(), qs, Hq, k.data_ptr(), ks, Hk, cos.data_ptr(), sin.data_ptr(), cs, B, S, D,
                        int(backward), qo.data_ptr(), ko.data_ptr(), _stream(q)))
    return qo, ko


def swiglu_fwd(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up for [rows, F] operands."""
    _require_cuda(gate, up)
    gate, up = _rows_operand(gate), _rows_operand(up)
    rows, F = gate.shape
    y = torch.empty(rows, F, dtype=torch.bfloat16, device=gate.device)
    _check(_lib.vq_swiglu_fwd(gate.data_ptr(), gate.stride(0), up.data_ptr(), up.stride(0), rows, F, y.data_ptr(),
                              y.stride(0), _stream(gate)))
    return y


def swiglu_bwd(gate: torch.Tensor, up: torch.Tensor, dy: torch.Tensor, out: torch.Tensor | None = None):
    """(d gate, d up) of silu(gate) * up; with ``out`` ([rows, 2F] bf16,
    contiguous) both are written into it side by side and returned as views."""
    _require_cuda(gate, up, dy)
    gate, up, dy = _rows_operand(gate), _rows_operand(up), _rows_operand(dy)
    rows, F = gate.shape
    if out is not None:
        if out.dtype != torch.bfloat16 or tuple(out.shape) != (rows, 2 * F) or not out.is_contiguous():
            raise ValueError("swiglu_bwd: out must be a contiguous bf16 [rows, 2F] tensor")
        dg, du = out[:, :F], out[:, F:]
    else:
        dg = torch.empty(rows, F, dtype=torch.bfloat16, device=gate.device)
        du = torch.empty(rows, F, dtype=torch.bfloat16, device=gate.device)
    _check(_lib.vq_swiglu_bwd(gate.data_ptr(), gate.stride(0), up.data_ptr(), up.stride(0), dy.data_ptr(), dy.stride(0),
                              rows, F, dg.data_ptr(), du.data_ptr(), dg.stride(0), _stream(gate)))
    return dg, du

