"""B200 (sm_100a) block-scaled quantise / GEMM path for DeepSeek-V4-style MoE.

``kernel`` holds the drop-in ops (act_quant, fp4_act_quant, fp8_gemm,
fp4_gemm, sparse_attn, hc_split_sinkhorn, and the Indexer's indexer_topk);
``moe`` the grouped per-expert MoE layer and its gate; ``ep`` and ``tp`` the
expert-parallel and tensor-parallel forms; ``loader`` the checkpoint
conversion into the kernel-native layout.  All compute runs in the CUDA
library ``libbsgemm.so`` built from ``csrc/`` (C ABI: include/bsgemm.h).
"""

from . import _lib  # noqa: F401
from .kernel import (act_quant, fp4_act_quant, fp8_gemm, fp4_gemm, sparse_attn, hc_split_sinkhorn,  # noqa: F401
                     indexer_topk, profile_report)

__all__ = ["act_quant", "fp4_act_quant", "fp8_gemm", "fp4_gemm", "sparse_attn", "hc_split_sinkhorn", "indexer_topk",
           "profile_report"]
