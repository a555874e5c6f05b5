"""CPU oracle for the quantized decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain torch CPU code, the reference algorithms the
B200 kernels replace.  It exists to check the CUDA path; it is imported only by
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py``.  The product (``local_kimi_b200``) never imports it and has no
CPU fallback.

Parity pinning: ``tests/test_oracle_golden.py`` checks every function here
against golden vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference package and records its
outputs at group size 32) and against the known answers of the reference's own
tests.  The group-128 codec is the same code with the group size as a
parameter; at group 32 it reproduces the reference bit for bit.

Modules:
  codec   quantise / dequantise / decode (engine/quant/w4a16.py:68-129)
  ops     dense, grouped, SwiGLU, down+combine, fused QKV, router, KDA step
  moe     one MoE decode layer in the reference's grouped structure
  synth   seeded synthetic inputs with BASELINE's shapes and distributions
"""
