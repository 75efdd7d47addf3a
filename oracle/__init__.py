"""CPU oracle for the MXFP4 quantized-expert path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the algorithm of the reference project
(sjdthree/kimi-k3-mlx-macmini) for its quantized-expert hot path:

* ``mxfp4_oracle`` (numpy): the MXFP4 codec, the sigmoid top-k router, one expert's
  SwiGLU/situ FFN and the whole MoE block with its weighted scatter-add.
* ``matvec_ref.c`` (plain C, built into ``_build/libk3oracle.so``): the reference's
  fused Metal kernel loop (sequential fp32 ``fma`` over k), used as the exact-order
  numeric check and as the timed CPU baseline.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline and
``--impl reference`` legs) may import this package, and only as the checker. The
product path (``kimi_k3_mlx_macmini_b200``) never imports it and has no CPU
fallback.

Parity pinning: every function here is checked against golden vectors produced by
the reference's own code (``k3ref``, ``tools/make_synthetic_k3.py``) and by the
third-party decoder it was proven against (``compressed_tensors``); see
``tests/golden/make_golden.py`` and ``tests/test_oracle.py``.
"""
