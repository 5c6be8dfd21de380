"""CPU oracle for the KernelForge hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline. The product (``kernelo_b200``) never
imports it and has no CPU fallback.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own code
(``kernelforge`` imported from its source tree, including its Triton kernels
under ``TRITON_INTERPRET=1`` for fp16/fp32) on seeded inputs and stores the
results as fixtures; ``tests/test_oracle.py`` checks this oracle against every
fixture and against the reference tests' known-answer pins.
"""

from oracle.cpu_reference import (  # noqa: F401
    gelu_erf,
    gelu_tanh,
    gemv_ref,
    linear_gelu_ref,
    matmul_ref,
    rmsnorm_ref,
    softmax_ref,
    torch_cpu,
)
