"""CPU oracle for the block-scaled GEMM path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy with explicit bit-level rounding, the PyTorch
CPU path of the reference module ``kernel_sm121.py`` (act_quant,
fp4_act_quant, _e8m0_to_fp32, fp8_gemm, fp4_gemm) plus a composed MoE layer
built from those ops.  It is the checker the parity tests compare the CUDA
kernels against; it is pinned against golden vectors that were produced by
running the reference itself (``tests/golden/make_golden.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import it.  The product path never routes through this package and
fails loudly when its CUDA extension is missing.
"""

from .blockscaled import *  # noqa: F401,F403
