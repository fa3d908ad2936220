"""The reference's CPU arithmetic, restated with torch on the host cores.

Test and baseline infrastructure only: ``bench.py`` times it as the
reference arm and as ``cpu_baseline`` (the reference project itself is a
Python module that is not installed on the GPU hosts), and
``tests/test_torch_cpu.py`` pins it against the golden vectors that the
reference produced.  Nothing on the product path imports it.

It follows the CPU branches of ``kernel_sm121.py`` step by step, with the
same torch operations and dtypes, so that it also runs at the reference's
speed: quantisation in fp32 tensor ops, and each GEMM as "dequantise both
operands in fp32, round them to bf16, one bf16 ``torch.mm``".

  act_quant  kernel_sm121.py:51-87
  fp8_gemm   kernel_sm121.py:236-251
  fp4_gemm   kernel_sm121.py:263-266 (code table), 334-340 (decode), 395-417
  e8m0       kernel_sm121.py:131-133

``moe_experts`` composes those ops into the MoE expert loop the reference's
caller runs (one act_quant and three fp4_gemm per active expert; the caller
is in DeepSeek's model file, outside the reference project).
"""

from __future__ import annotations

import torch

__all__ = ["act_quant", "fp8_gemm", "fp4_gemm", "e8m0_to_f32", "moe_experts"]

# e2m1 code -> value; codes 9..15 are the negatives of 1..7 and code 8 (-0)
# decodes to +0.0, as in the reference's table
_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                      0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float32)


def e8m0_to_f32(s: torch.Tensor) -> torch.Tensor:
    """e8m0 byte b -> float with exponent field b (b=0 gives 0.0, 255 gives inf)."""
    return (s.view(torch.uint8).to(torch.int32) << 23).view(torch.float32)


def _scales(s: torch.Tensor) -> torch.Tensor:
    return e8m0_to_f32(s) if s.dtype in (torch.float8_e8m0fnu, torch.uint8) else s.float()


def act_quant(x: torch.Tensor, block_size: int = 128, pow2: bool = False):
    """Per 1 x block_size block of the last dim: s = max(amax, 1e-4) / 448
    (rounded up to a power of two when ``pow2``); y = e4m3(clamp(x / s))."""
    K = x.size(-1)
    blk = x.reshape(-1, K // block_size, block_size).float()
    s = blk.abs().amax(dim=-1).clamp(min=1e-4) / 448.0
    if pow2:
        s = torch.exp2(torch.ceil(torch.log2(s)))
    y = (blk / s[..., None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return y.reshape(x.shape), s.reshape(*x.shape[:-1], K // block_size)


def _rows_bf16(a: torch.Tensor, a_s: torch.Tensor) -> torch.Tensor:
    """e4m3 [M, K] times its 1x128 scales, rounded to bf16."""
    M, K = a.shape
    return (a.float().view(M, K // 128, 128) * _scales(a_s).view(M, K // 128, 1)).view(M, K).to(torch.bfloat16)


def fp8_gemm(a: torch.Tensor, a_s: torch.Tensor, b: torch.Tensor, b_s: torch.Tensor) -> torch.Tensor:
    """C = A @ B^T; A e4m3 [M, K] with 1x128 scales, B e4m3 [N, K] with
    128x128 block scales [ceil(N/128), K/128]; bf16 out."""
    M, K = a.shape
    N = b.shape[0]
    bs = _scales(b_s).repeat_interleave(128, dim=0)[:N]                     # [N, K/128]
    b_deq = (b.float().view(N, K // 128, 128) * bs[..., None]).view(N, K).to(torch.bfloat16)
    return torch.mm(_rows_bf16(a, a_s), b_deq.t())


def fp4_gemm(a: torch.Tensor, a_s: torch.Tensor, b: torch.Tensor, b_s: torch.Tensor) -> torch.Tensor:
    """C = A @ B^T; A e4m3 [M, K] with 1x128 scales, B packed e2m1 [N, K/2]
    (low nibble = even k) with 1x32 scales; bf16 out.  All of B is decoded
    on every call, as in the reference's CPU branch."""
    M, K = a.shape
    N = b.shape[0]
    raw = b.view(torch.uint8).long()
    vals = torch.stack([_E2M1[raw & 0xF], _E2M1[raw >> 4]], dim=-1).view(N, K // 32, 32)
    b_deq = (vals * _scales(b_s).view(N, K // 32, 1)).view(N, K).to(torch.bfloat16)
    return torch.mm(_rows_bf16(a, a_s), b_deq.t())


def moe_experts(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, experts, w13, w13_s, w2, w2_s,
                out: torch.Tensor) -> None:
    """Adds the listed experts' weighted outputs into ``out`` (fp32 [T, H]).

    Per expert e and the tokens routed to it: h = act_quant(x, ue8m0);
    g, u = fp4_gemm(h, W1_e), fp4_gemm(h, W3_e) (W13_e rows [0, I) and
    [I, 2I)); z = silu(g) * u in fp32; y = fp4_gemm(act_quant(z, ue8m0),
    W2_e); out[t] += w[t, slot] * y.  ``w13[e]`` etc. may be fetched lazily.
    """
    for e in experts:
        tok, slot = torch.nonzero(idx == e, as_tuple=True)
        if tok.numel() == 0:
            continue
        h, hs = act_quant(x[tok], 128, pow2=True)
        W13, W13s = w13[e], w13_s[e]
        inter = W13.shape[0] // 2
        g = fp4_gemm(h, hs, W13[:inter], W13s[:inter]).float()
        u = fp4_gemm(h, hs, W13[inter:], W13s[inter:]).float()
        q, qs = act_quant(torch.nn.functional.silu(g) * u, 128, pow2=True)
        y = fp4_gemm(q, qs, w2[e], w2_s[e]).float()
        out.index_add_(0, tok, w[tok, slot, None] * y)
