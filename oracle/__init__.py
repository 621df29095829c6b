"""CPU oracle for the GLAD INT8 rollout forward -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, what the reference's qrt INT8 path computes
(every function cites the reference file:line it follows). It is the checker:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import it. The product (``rl_quant_b200``) never calls it, and the
product path fails loudly when its CUDA library is missing.

Parity pinning: ``tests/test_oracle.py`` checks this oracle against golden
vectors produced by running the reference itself (rsl_rl + qrt, with the two
Triton kernels of ``qrt/qconv.py`` executed by Triton's CPU interpreter); see
``tests/golden/make_golden.py``.
"""
