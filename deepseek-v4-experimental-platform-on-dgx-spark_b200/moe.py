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

__all__ = ["moe_forward", "gate_logits", "MoEWeights", "MoEWorkspace", "pack_scales"]


def pack_scales(w_s: torch.Tensor) -> torch.Tensor:
    """ue8m0 weight scales [E, rows, K/32] -> the packed tcgen05 chunk layout
    [E][rows/128][K/128][512 B] (same byte count), once at weight-load time."""
    E, rows, kq = w_s.shape
    src = w_s.contiguous().view(torch.uint8)
    out = torch.empty(E * rows * kq, dtype=torch.uint8, device=w_s.device)
    _lib.check(_lib.load().bs_moe_pack_scales(src.data_ptr(), E, rows, kq * 32, out.data_ptr(),
                                              torch.cuda.current_stream(w_s.device).cuda_stream))
    return out


class MoEWeights:
    """One MoE layer's expert weights in kernel-native form.

    w13 [E, 2I, H/2] and w2 [E, H, I/2] stay as given (packed e2m1 bytes);
    their ue8m0 scales are re-laid out once by :func:`pack_scales`.
    """

    def __init__(self, w13: torch.Tensor, w13_s: torch.Tensor, w2: torch.Tensor, w2_s: torch.Tensor):
        if not (w13.is_cuda and w2.is_cuda):
            raise RuntimeError("MoEWeights must live on a CUDA device")
        self.E, two_i, h_half = w13.shape
        self.I, self.H = two_i // 2, h_half * 2
        if tuple(w2.shape) != (self.E, self.H, self.I // 2):
            raise ValueError(f"w2 shape {tuple(w2.shape)} does not match w13 {tuple(w13.shape)}")
        if tuple(w13_s.shape) != (self.E, two_i, self.H // 32) or tuple(w2_s.shape) != (self.E, self.H, self.I // 32):
            raise ValueError("scale shapes do not match the weights")
        self.w13 = w13.contiguous().view(torch.uint8)
        self.w2 = w2.contiguous().view(torch.uint8)
        self.w13_sp = pack_scales(w13_s)
        self.w2_sp = pack_scales(w2_s)


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


def gate_logits(x: torch.Tensor, gate_weight: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Gate projection on the tensor cores: x bf16 [T, H] . gate_weight bf16
    [E, H]^T -> fp32 logits [T, E] (the routing input of moe_forward)."""
    if not (x.is_cuda and gate_weight.is_cuda):
        raise RuntimeError("gate_logits runs on CUDA tensors only (no CPU fallback)")
    if x.dtype != torch.bfloat16 or gate_weight.dtype != torch.bfloat16:
        raise TypeError("gate_logits expects bf16 activations and gate weights")
    T, H = x.shape
    E = gate_weight.shape[0]
    if gate_weight.shape[1] != H:
        raise ValueError(f"gate weight {tuple(gate_weight.shape)} does not match hidden {H}")
    if out is None:
        out = torch.empty(T, E, dtype=torch.float32, device=x.device)
    xc, wc = x.contiguous(), gate_weight.contiguous()
    _lib.check(_lib.load().bs_moe_gate(xc.data_ptr(), wc.data_ptr(), T, E, H, out.data_ptr(),
                                       torch.cuda.current_stream(x.device).cuda_stream))
    return out


def moe_forward(x: torch.Tensor, logits: torch.Tensor | None, weights: MoEWeights, topk: int,
                out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                gate_weight: torch.Tensor | None = None) -> torch.Tensor:
    """MoE layer: x bf16 [T, H], logits fp32 [T, E] -> bf16 [T, H].  With
    ``gate_weight`` (bf16 [E, H]) instead of logits, the gate projection runs
    first on the device (gate_logits), then the same layer."""
    if logits is None:
        if gate_weight is None:
            raise ValueError("moe_forward needs gate logits or a gate weight")
        logits = gate_logits(x, gate_weight)
    if not (x.is_cuda and logits.is_cuda):
        raise RuntimeError("moe_forward runs on CUDA tensors only (no CPU fallback)")
    T, H = x.shape
    E = logits.shape[1]
    if x.dtype != torch.bfloat16 or logits.dtype != torch.float32:
        raise TypeError("moe_forward expects bf16 activations and fp32 logits")
    if (E, H) != (weights.E, weights.H):
        raise ValueError(f"moe_forward: x/logits ({H}, {E}) do not match the weights ({weights.H}, {weights.E})")
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        workspace = _WS.get(x.device, T, H, weights.I, E, topk)
    lib = _lib.load()
    xc, lc = x.contiguous(), logits.contiguous()
    _lib.check(lib.bs_moe_forward(xc.data_ptr(), lc.data_ptr(), T, H, weights.I, E, topk, weights.w13.data_ptr(),
                                  weights.w13_sp.data_ptr(), weights.w2.data_ptr(), weights.w2_sp.data_ptr(),
                                  out.data_ptr(), workspace.data_ptr(), workspace.numel(),
                                  torch.cuda.current_stream(x.device).cuda_stream))
    return out
