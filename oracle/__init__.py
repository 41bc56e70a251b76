"""CPU oracle for the vates_b200 hot path.

TEST INFRASTRUCTURE ONLY. This package restates, on the CPU, the arithmetic
that AMOS144/Vates runs on its hot path (fused quantized MoE, pool slot-table
gather, IsoQuant K4/V3 KV quantize + attend). It exists so that tests, the
``smoke()`` check and the ``cpu_baseline`` leg of ``bench.py`` have something to
compare the CUDA kernels against. Nothing in the ``vates_b200`` product package
imports it, and the product path never falls back to it.

Where the reference's arithmetic lives in MLX 0.31.2 / mlx-lm 0.31.3 (pinned in
the reference's ``uv.lock:320-322, 350-352``; neither is vendored and MLX cannot
be installed here), the published algorithm of the MLX op is restated and the
reference call site is cited next to each function.

Parity pins:
- ``build_block_so4`` is pinned bit-exactly against the reference's own
  ``mlx_streaming/core/cache/quant_kv.py:24-65`` run in this container with a
  numpy stand-in for ``mlx.core`` (fixtures in ``tests/golden``).
- ``route_reduce`` is pinned against the hand-computed expectations of
  ``mlx_streaming/tests/test_expert_major_prefill.py:89-132``.
- ``mlx_affine_quantize`` / quantized-matmul rounding points follow MLX's
  published source; no MLX run is available to pin them (parity against MLX
  itself is unpinned for those codes).
"""
