"""Voodoo dynamic quantisation -- B200-native gated-candidate training step.

Same package name and module layout as the reference (curvedinf/voodoo-dyn-quant)
for the hot path it replaces:

- :mod:`voodoo_quant.ggml`      quant-type registry, libggml quantisation boundary
- :mod:`voodoo_quant.cache`     compile-cache setup + HBM-resident packed candidate arenas
- :mod:`voodoo_quant.layers`    MixedQuantLinear / MixedQuantEmbedding on the sm_100a kernels
- :mod:`voodoo_quant.parallel`  tensor parallelism (NCCL over NVLink)
- :mod:`voodoo_quant.training`  fused distillation loss
- :mod:`voodoo_quant._C`        ctypes binding of libvoodoo_b200.so
"""

from voodoo_quant.cache import setup_caches  # noqa: F401

__version__ = "0.1.0+b200"
