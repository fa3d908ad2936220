"""Grouped per-expert MoE layer on one GPU (the hot path's MoE form).

The reference runs experts one by one from DeepSeek's model code: for each
expert with routed tokens, ``act_quant`` then ``fp4_gemm`` with W1 and W3,
SwiGLU, ``act_quant`` and ``fp4_gemm`` with W2, then a weighted sum over the
top-k experts (DevHistory.md:557, 754 of the reference describe the loop;
the loop itself lives in the external model file).  Here the whole layer is
one call into the CUDA library: routing, histogram, expert-sorted dispatch,
two persistent grouped tcgen05 GEMMs (the first with a fused SwiGLU + e4m3
quantisation epilogue) and a deterministic combine -- no host sync.

Weight layout per expert e (packed e2m1, two codes per byte, low nibble =
even k; ue8m0 scales per 1x32):
  w13  [E, 2*I, H/2], w13_s [E, 2*I, H/32]   rows [0,I) = W1 (gate), [I,2I) = W3 (up)
  w2   [E, H, I/2],   w2_s  [E, H, I/32]
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["moe_forward", "MoEWorkspace"]


class MoEWorkspace:
    """Caches one device workspace per (device, T, H, I, E, topk)."""

    def __init__(self):
        self._bufs = {}

    def get(self, device, T, H, I, E, topk) -> torch.Tensor:
        key = (str(device), T, H, I, E, topk)
        buf = self._bufs.get(key)
        if buf is None:
            n = _lib.load().bs_moe_workspace_size(T, H, I, E, topk)
            if n == 0:
                raise NotImplementedError(f"moe: unsupported sizes T={T} H={H} I={I} E={E} topk={topk}")
            buf = torch.empty(n, dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf


_WS = MoEWorkspace()


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.uint8)


def moe_forward(x: torch.Tensor, logits: torch.Tensor, w13: torch.Tensor, w13_s: torch.Tensor, w2: torch.Tensor,
                w2_s: torch.Tensor, topk: int, out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """MoE layer: x bf16 [T, H], logits fp32 [T, E] -> bf16 [T, H]."""
    if not (x.is_cuda and logits.is_cuda and w13.is_cuda and w2.is_cuda):
        raise RuntimeError("moe_forward runs on CUDA tensors only (no CPU fallback)")
    T, H = x.shape
    E = logits.shape[1]
    I = w2.shape[2] * 2
    if x.dtype != torch.bfloat16 or logits.dtype != torch.float32:
        raise TypeError("moe_forward expects bf16 activations and fp32 logits")
    if tuple(w13.shape) != (E, 2 * I, H // 2) or tuple(w2.shape) != (E, H, I // 2):
        raise ValueError(f"moe_forward: weight shapes {tuple(w13.shape)} / {tuple(w2.shape)} do not match "
                         f"E={E}, H={H}, I={I}")
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        workspace = _WS.get(x.device, T, H, I, E, topk)
    lib = _lib.load()
    xc, lc = x.contiguous(), logits.contiguous()
    w13u, w13s, w2u, w2s = _u8(w13), _u8(w13_s), _u8(w2), _u8(w2_s)
    _lib.check(lib.bs_moe_forward(xc.data_ptr(), lc.data_ptr(), T, H, I, E, topk, w13u.data_ptr(),
                                  w13s.data_ptr(), w2u.data_ptr(), w2s.data_ptr(), out.data_ptr(),
                                  workspace.data_ptr(), workspace.numel(),
                                  torch.cuda.current_stream(x.device).cuda_stream))
    return out
