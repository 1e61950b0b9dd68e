"""CPU oracle for the FAQUANT HiF4 hot paths -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference algorithms the CUDA kernels of
``faquant_b200`` must reproduce:

- ``oracle.hif4``: the HiF4 S1P2 quantizer of ``src/faquant/hif4.py``;
- ``oracle.rotation``: the Walsh-Hadamard / block-Hadamard / HiSQ input rotation
  of ``src/faquant/rotation.py`` and ``src/faquant/hisq_rotation.py``;
- ``oracle.linear``: ``FakeQuantLinear.forward`` of ``src/faquant/quantization.py``;
- ``oracle.attention``: the tiled HiF4 attention simulator of
  ``src/faquant/simulated_flash_attention.py`` and the post-RoPE Q/K transform of
  ``src/faquant/qwen3.py``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the
checker or the timed CPU baseline. The product path (``faquant_b200``) never
imports it and has no CPU fallback.

Parity pin: the three-level HiF4 quantizer is pinned to the upstream
GCC-HiFloat golden vector held by the reference test
``tests/test_quantization.py:51-74`` (fixture ``tests/golden/hif4_golden.npz``);
every other function is pinned to outputs of the reference itself, imported
in the build container by ``tests/golden/make_golden.py``. The two-level
``12``/``13`` variants have no upstream golden vector: they are pinned to the
reference implementation only.
"""
