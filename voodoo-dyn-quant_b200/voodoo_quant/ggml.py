"""GGUF quant-type registry and the libggml quantisation boundary.

Same public surface as the reference module (voodoo_quant/ggml.py:30-281):
``QuantTypeInfo``, ``_QUANT_REGISTRY``, ``QUANT_LADDER``, ``find_libggml``,
``lib_path``, ``list_quant_types``, ``default_candidate_types``,
``get_quant_info``, ``bytes_per_weight``, ``quantize_tensor``,
``dequantize_tensor``, ``estimate_bytes``.

Differences, all additive:

* The registry gains Q2_K (ggml type 10, 256 weights, 84 bytes) and Q3_K
  (type 11, 256, 110), which the benchmark candidate menus need and the
  reference lacks.
* ``dequantize_tensor`` of a CUDA tensor runs the bit-exact sm_100a decoder of
  libvoodoo_b200 (``_C.dequant``); CPU tensors still go to libggml exactly as
  in the reference.  ``quantize_tensor`` is unchanged: llama.cpp's own
  quantiser through ctypes.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np
import torch

QK_K = 256


class QuantTypeInfo:
    def __init__(self, name: str, ggml_type: int, block_size: int, block_bytes: int, quant_func: str,
                 dequant_func: str):
        self.name = name
        self.ggml_type = ggml_type
        self.block_size = block_size
        self.block_bytes = block_bytes
        self.quant_func = quant_func
        self.dequant_func = dequant_func

    def bytes_per_weight(self) -> float:
        return self.block_bytes / self.block_size


def _info(name: str, tid: int, bs: int, bb: int) -> QuantTypeInfo:
    # ggml symbol names: quantize_q4_K / dequantize_row_q4_K, quantize_iq4_xs, ...
    stem = name.lower() if name.startswith(("IQ", "TQ")) else "q" + name[1:]
    return QuantTypeInfo(name, tid, bs, bb, f"quantize_{stem}", f"dequantize_row_{stem}")


_QUANT_REGISTRY: dict[str, QuantTypeInfo] = {
    n: _info(n, t, bs, bb)
    for n, t, bs, bb in (
        ("IQ1_S", 19, 256, 50), ("IQ1_M", 29, 256, 56), ("IQ2_XXS", 16, 256, 66), ("IQ2_XS", 17, 256, 74),
        ("IQ2_S", 22, 256, 82), ("IQ3_XXS", 18, 256, 98), ("IQ3_S", 21, 256, 110), ("IQ4_XS", 23, 256, 136),
        ("Q2_K", 10, 256, 84), ("Q3_K", 11, 256, 110),
        ("Q4_K", 12, 256, 144), ("Q5_K", 13, 256, 176), ("Q6_K", 14, 256, 210), ("Q8_0", 8, 32, 34),
        ("TQ1_0", 34, 256, 54), ("TQ2_0", 35, 256, 66),
    )
}

# Formats with a B200 decoder (all BASELINE candidate menus fall inside it).
GPU_FORMATS = ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0", "IQ4_XS")

QUANT_LADDER: list[str] = [
    "IQ1_S", "IQ1_M", "IQ2_XXS", "IQ2_XS", "IQ2_S", "Q2_K",
    "IQ3_XXS", "IQ3_S", "Q3_K", "IQ4_XS", "Q4_K", "Q5_K", "Q6_K", "Q8_0",
]

_LIB_NAME = "libggml-base.so"
_LIB: "ctypes.CDLL | None" = None


def _candidate_paths() -> list[Path]:
    paths: list[Path] = []
    env = os.environ.get("VOODOO_GGML_LIB")
    if env:
        paths.append(Path(env))
    repo_root = Path(__file__).resolve().parent.parent
    paths.append(repo_root / "third_party" / "llama.cpp" / "build" / "bin" / _LIB_NAME)
    for sibling in sorted(repo_root.parent.glob("llama.cpp*")):
        paths.append(sibling / "build" / "bin" / _LIB_NAME)
    return paths


def find_libggml() -> Path | None:
    for p in _candidate_paths():
        if p.exists():
            return p
    try:
        ctypes.CDLL(_LIB_NAME)
        return Path(_LIB_NAME)
    except OSError:
        return None


def _load_lib() -> "ctypes.CDLL":
    global _LIB
    if _LIB is not None:
        return _LIB
    found = find_libggml()
    if found is None:
        raise RuntimeError(
            "libggml-base.so not found. Run `make llamacpp` (builds into third_party/), "
            "or set VOODOO_GGML_LIB=/path/to/libggml-base.so, or install llama.cpp system-wide."
        )
    try:
        lib = ctypes.CDLL(str(found))
    except OSError:
        raise RuntimeError(f"Failed to load libggml-base from {found}.") from None
    lib.ggml_quantize_init.argtypes = [ctypes.c_int]
    lib.ggml_quantize_init.restype = None
    for info in _QUANT_REGISTRY.values():
        q = getattr(lib, info.quant_func, None)
        if q is not None:
            q.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                          ctypes.POINTER(ctypes.c_float)]
            q.restype = ctypes.c_size_t
        d = getattr(lib, info.dequant_func, None)
        if d is not None:
            d.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int64]
            d.restype = None
    _LIB = lib
    return lib


def lib_path() -> str | None:
    p = find_libggml()
    return str(p) if p else None


def list_quant_types() -> list[str]:
    return list(_QUANT_REGISTRY.keys())


def default_candidate_types() -> list[str]:
    return [qt for qt in list_quant_types() if not qt.startswith("TQ")]


def get_quant_info(quant_type: str) -> QuantTypeInfo:
    if quant_type not in _QUANT_REGISTRY:
        raise ValueError(f"Unknown quant type: {quant_type}. Supported: {list(_QUANT_REGISTRY.keys())}")
    return _QUANT_REGISTRY[quant_type]


def bytes_per_weight(quant_type: str) -> float:
    return get_quant_info(quant_type).bytes_per_weight()


def quantize_tensor(weight: torch.Tensor, quant_type: str, imatrix: torch.Tensor | None = None) -> torch.Tensor:
    """llama.cpp quantiser (libggml-base via ctypes) -> uint8 [nblocks, block_bytes].

    A CUDA weight quantised to Q8_0 without an importance matrix takes the
    sm_100a quantiser instead (``vq_quantize``: ggml's reference Q8_0 rule,
    byte-identical) and the result stays on that device."""
    info = get_quant_info(quant_type)
    if weight.is_cuda and quant_type == "Q8_0" and imatrix is None:
        from voodoo_quant import _C

        w = weight.detach()
        if w.dim() != 2:
            raise ValueError(f"quantize_tensor expects a 2-D weight, got shape {tuple(w.shape)}")
        return _C.quantize(w, "Q8_0")
    weight = weight.detach().to("cpu", torch.float32).contiguous()
    out_features, in_features = weight.shape
    if in_features % info.block_size != 0:
        raise ValueError(f"{quant_type} requires in_features % {info.block_size} == 0, got {in_features}")
    lib = _load_lib()
    lib.ggml_quantize_init(info.ggml_type)
    nb = out_features * (in_features // info.block_size)
    out_bytes = nb * info.block_bytes
    if imatrix is None:
        imatrix = torch.ones(in_features, dtype=torch.float32)
    imatrix = imatrix.to(torch.float32).contiguous()
    if imatrix.numel() != in_features:
        raise ValueError(f"imatrix size {imatrix.numel()} != in_features {in_features}")
    dst = (ctypes.c_uint8 * out_bytes)()
    res = getattr(lib, info.quant_func)(
        ctypes.cast(weight.data_ptr(), ctypes.POINTER(ctypes.c_float)), ctypes.byref(dst), out_features,
        in_features, ctypes.cast(imatrix.data_ptr(), ctypes.POINTER(ctypes.c_float)))
    if res != out_bytes:
        raise RuntimeError(f"{info.quant_func} returned {res} bytes, expected {out_bytes}")
    return torch.from_numpy(np.frombuffer(bytes(dst), dtype=np.uint8).copy()).reshape(nb, info.block_bytes)


def dequantize_tensor(qweight: torch.Tensor, quant_type: str, out_features: int, in_features: int,
                      pin_memory: bool = False) -> torch.Tensor:
    """Packed blocks -> float32 [out_features, in_features].

    CUDA tensors: bit-exact sm_100a decoder.  CPU tensors: libggml, as in the
    reference (ggml.py:224-269).
    """
    info = get_quant_info(quant_type)
    if in_features % info.block_size != 0:
        raise ValueError(f"{quant_type} requires in_features % {info.block_size} == 0, got {in_features}")
    nb = out_features * (in_features // info.block_size)
    if qweight.numel() != nb * info.block_bytes:
        raise ValueError(
            f"qweight size {qweight.numel()} does not match {nb} blocks of {info.block_bytes} bytes for {quant_type}")
    if qweight.is_cuda:
        if quant_type not in GPU_FORMATS:
            raise ValueError(f"{quant_type} has no B200 decoder; supported: {list(GPU_FORMATS)}")
        from voodoo_quant import _C
        return _C.dequant(qweight, quant_type, out_features, in_features)
    lib = _load_lib()
    qweight = qweight.reshape(nb, info.block_bytes).contiguous()
    out = torch.empty(out_features * in_features, dtype=torch.float32, pin_memory=pin_memory)
    getattr(lib, info.dequant_func)(ctypes.cast(qweight.data_ptr(), ctypes.c_void_p),
                                    ctypes.cast(out.data_ptr(), ctypes.POINTER(ctypes.c_float)),
                                    out_features * in_features)
    return out.reshape(out_features, in_features)


def estimate_bytes(shape: tuple[int, ...], quant_type: str | None, source_dtype: torch.dtype = torch.bfloat16) -> int:
    numel = int(np.prod(shape))
    if quant_type is None:
        return numel * torch.finfo(source_dtype).bits // 8
    return int(numel * bytes_per_weight(quant_type))
