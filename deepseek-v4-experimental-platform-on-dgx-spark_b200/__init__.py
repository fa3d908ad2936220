"""B200 (sm_100a) block-scaled quantise / GEMM path for DeepSeek-V4-style MoE.

``kernel`` holds the drop-in ops (act_quant, fp4_act_quant, fp8_gemm,
fp4_gemm); ``moe`` the grouped per-expert MoE layer; ``ep`` and ``tp`` the
expert-parallel and tensor-parallel forms.  All compute runs in the CUDA
library ``libbsgemm.so`` built from ``csrc/`` (C ABI: include/bsgemm.h).
"""

from . import _lib  # noqa: F401
from .kernel import act_quant, fp4_act_quant, fp8_gemm, fp4_gemm, profile_report  # noqa: F401

__all__ = ["act_quant", "fp4_act_quant", "fp8_gemm", "fp4_gemm", "profile_report"]
