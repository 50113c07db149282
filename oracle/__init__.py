"""CPU oracle for the gated-candidate training step -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy, the arithmetic of the reference
(curvedinf/voodoo-dyn-quant) on the gated-Linear hot path:

* ``ggml_blocks`` -- per-format GGUF block decoding (Q2_K, Q3_K, Q4_K, Q5_K,
  Q6_K, Q8_0, IQ4_XS), operation-for-operation in the order the reference's
  torch decoders use, so float32 results are bit-identical.
* ``mixgemm``     -- the softmax candidate mixture, the forward/backward GEMMs
  and the gate gradient <dY^T X, W_k> in float32/float64.
* ``loss``        -- cross entropy + lambda * T^2 * KL(teacher || student) and
  its gradient with respect to the student logits.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline.  The product path (``voodoo_quant``)
never imports it and fails loudly when its CUDA library is missing.

Parity pin: ``tests/golden/`` holds vectors produced by the reference's own
torch decoders (``voodoo_quant/layers.py:62-213``,
``voodoo_quant/quants/gpu_dequant.py:460-519``) and by gguf-py 0.19.0 (the
reference's declared dependency, ``pyproject.toml:24``) for Q2_K/Q3_K, which the
reference itself cannot decode; ``tests/test_oracle_golden.py`` checks this
oracle against them bit for bit.
"""
