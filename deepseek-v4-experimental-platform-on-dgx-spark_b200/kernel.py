"""Drop-in replacement for the block-scaled ops of the reference's ``kernel`` module.

The reference (``kernel_sm121.py``) is injected as ``sys.modules['kernel']``
and DeepSeek's model code does ``from kernel import act_quant, fp4_act_quant,
fp8_gemm, fp4_gemm, ...``.  This module keeps those four signatures, defaults,
return conventions and error behaviour, and runs every call through the
sm_100a CUDA library (``libbsgemm.so``, C ABI in ``include/bsgemm.h``):

  act_quant(x, block_size=128, scale_fmt=None, scale_dtype=torch.float32, inplace=False)
  fp4_act_quant(x, block_size=32, inplace=False)
  fp8_gemm(a, a_s, b, b_s, scale_dtype=torch.float32)
  fp4_gemm(a, a_s, b, b_s, scale_dtype=torch.float32)

CPU tensors are an error: there is no CPU fallback here.
"""

from __future__ import annotations

import time as _time
from typing import Optional

import torch

from . import _lib

__all__ = ["act_quant", "fp4_act_quant", "fp8_gemm", "fp4_gemm", "sparse_attn", "hc_split_sinkhorn", "indexer_topk",
           "profile_report"]

# Per-op call counter and host-side seconds, reported by profile_report() in
# the same columns as the reference module's report (kernel_sm121.py:31-44).
# The host clock brackets the launch only (no device sync), so for these
# asynchronous kernels it measures launch cost, as the reference's does.
_PROFILE: dict = {}


def _tally(op: str, t0: float) -> None:
    rec = _PROFILE.setdefault(op, [0, 0.0])
    rec[0] += 1
    rec[1] += _time.perf_counter() - t0


def profile_report():
    """Print each op's call count and host seconds (largest first), then clear them."""
    if not _PROFILE:
        return
    rows = sorted(_PROFILE.items(), key=lambda item: item[1][1], reverse=True)
    secs = sum(rec[1] for _, rec in rows)
    calls = sum(rec[0] for _, rec in rows)
    lines = ["[bsgemm] per-op host time"]
    for op, (n, t) in rows:
        share = 100.0 * t / secs if secs > 0 else 0.0
        lines.append(f"  {op:25s}: {n:6d} calls, {t:7.3f}s ({share:5.1f}%)")
    lines.append(f"  {'TOTAL':25s}: {calls:6d} calls, {secs:7.3f}s")
    print("\n".join(lines), flush=True)
    _PROFILE.clear()


_X_DT = {torch.bfloat16: _lib.DT_BF16, torch.float16: _lib.DT_F16, torch.float32: _lib.DT_F32}
_S_DT = {torch.float32: _lib.DT_F32, torch.bfloat16: _lib.DT_BF16, torch.float16: _lib.DT_F16,
         torch.float8_e8m0fnu: _lib.DT_E8M0}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("bsgemm ops run on CUDA tensors only (no CPU fallback)")


def act_quant(x: torch.Tensor, block_size: int = 128, scale_fmt: Optional[str] = None,
              scale_dtype: torch.dtype = torch.float32, inplace: bool = False):
    """Block-wise e4m3 quantisation (kernel_sm121.py:55-87).

    Returns ``(y, s)`` with ``y`` float8_e4m3fn shaped like ``x`` and ``s``
    shaped ``[..., K/block_size]`` in ``scale_dtype``; with ``inplace=True``
    quantises-dequantises ``x`` in place and returns it.
    """
    t0 = _time.perf_counter()
    N = x.size(-1)
    assert N % block_size == 0
    _require_cuda(x)
    xc = x.contiguous()
    if xc.dtype not in _X_DT:
        xc = xc.float()
    rows = xc.numel() // N if N else 0
    lib = _lib.load()
    pow2 = 1 if scale_fmt is not None else 0
    if inplace:
        _lib.check(lib.bs_act_quant_inplace(xc.data_ptr(), _X_DT[xc.dtype], rows, N, block_size, pow2, _stream(x)))
        if xc.data_ptr() != x.data_ptr() or xc.dtype != x.dtype:
            x.copy_(xc)
        _tally("act_quant_inplace", t0)
        return x
    if scale_dtype not in _S_DT:
        raise NotImplementedError(f"act_quant: scale_dtype {scale_dtype} not supported")
    y = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(*x.shape[:-1], N // block_size, dtype=scale_dtype, device=x.device)
    _lib.check(lib.bs_act_quant(xc.data_ptr(), _X_DT[xc.dtype], rows, N, block_size, pow2, y.data_ptr(),
                                s.data_ptr(), _S_DT[scale_dtype], _stream(x)))
    _tally("act_quant", t0)
    return y, s


def fp4_act_quant(x: torch.Tensor, block_size: int = 32, inplace: bool = False) -> torch.Tensor:
    """In-place e2m1 fake quantisation (kernel_sm121.py:94-124)."""
    N = x.size(-1)
    assert N % block_size == 0
    if not inplace:
        raise NotImplementedError("fp4_act_quant: only inplace=True is supported (the model calls it in place)")
    _require_cuda(x)
    xc = x.contiguous()
    if xc.dtype not in _X_DT:
        xc = xc.float()
    rows = xc.numel() // N if N else 0
    _lib.check(_lib.load().bs_fp4_act_quant_inplace(xc.data_ptr(), _X_DT[xc.dtype], rows, N, block_size, _stream(x)))
    if xc.data_ptr() != x.data_ptr() or xc.dtype != x.dtype:
        x.copy_(xc)
    return x


def _scale_arg(s: torch.Tensor):
    """Scales as the library takes them: fp32 or raw e8m0 bytes."""
    if s.dtype == torch.float8_e8m0fnu:
        return s.contiguous(), _lib.DT_E8M0
    if s.dtype == torch.float32:
        return s.contiguous(), _lib.DT_F32
    return s.float().contiguous(), _lib.DT_F32


def fp8_gemm(a: torch.Tensor, a_s: torch.Tensor, b: torch.Tensor, b_s: torch.Tensor,
             scale_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """C[M,N] = A_e4m3[M,K] @ B_e4m3[N,K]^T with 1x128 / 128x128 block scales
    (kernel_sm121.py:190-255).  Returns bf16 shaped ``[..., N]``."""
    t0 = _time.perf_counter()
    K = a.size(-1)
    M = a.numel() // K
    N = b.size(0)
    out_shape = (*a.shape[:-1], N)
    _require_cuda(a, a_s, b, b_s)
    a_flat = a.view(M, K).contiguous()
    b_flat = b.contiguous()
    a_sf, as_dt = _scale_arg(a_s.view(M, -1))
    b_sf, bs_dt = _scale_arg(b_s)
    if a_flat.dtype != torch.float8_e4m3fn or b_flat.dtype != torch.float8_e4m3fn:
        raise TypeError("fp8_gemm expects float8_e4m3fn operands")
    if a_sf.shape != (M, K // 128) or b_sf.shape != ((N + 127) // 128, K // 128):
        raise ValueError(f"fp8_gemm: scale shapes {tuple(a_sf.shape)} / {tuple(b_sf.shape)} do not match "
                         f"M={M}, N={N}, K={K}")
    out = torch.empty(M, N, device=a.device, dtype=torch.bfloat16)
    _lib.check(_lib.load().bs_fp8_gemm(a_flat.data_ptr(), a_sf.data_ptr(), as_dt, b_flat.data_ptr(),
                                       b_sf.data_ptr(), bs_dt, M, N, K, out.data_ptr(), _stream(a)))
    _tally("fp8_gemm", t0)
    return out.view(out_shape)


def _fp4_gemm_fp32_scales(a_flat: torch.Tensor, a_sf: torch.Tensor, as_dt: int, b_u8: torch.Tensor,
                          b_s: torch.Tensor, M: int, N: int, K: int) -> torch.Tensor:
    """fp32 weight scales of any value: the reference CPU branch's arithmetic
    (kernel_sm121.py:402-417) -- both operands dequantised to bf16 on the
    device, then one bf16 GEMM with fp32 accumulation (torch.mm, a plain
    library GEMM).  No host sync."""
    lib = _lib.load()
    st = _stream(a_flat)
    bs = b_s.float().contiguous()
    if bs.shape != (N, K // 32):
        raise ValueError(f"fp4_gemm: weight scale shape {tuple(bs.shape)} does not match N={N}, K={K}")
    a_bf = torch.empty(M, K, dtype=torch.bfloat16, device=a_flat.device)
    b_bf = torch.empty(N, K, dtype=torch.bfloat16, device=a_flat.device)
    _lib.check(lib.bs_e4m3_rows_to_bf16(a_flat.data_ptr(), a_sf.data_ptr(), as_dt, M, K, a_bf.data_ptr(), st))
    _lib.check(lib.bs_fp4_weights_to_bf16(b_u8.data_ptr(), bs.data_ptr(), N, K, b_bf.data_ptr(), st))
    return torch.mm(a_bf, b_bf.t())


def fp4_gemm(a: torch.Tensor, a_s: torch.Tensor, b: torch.Tensor, b_s: torch.Tensor,
             scale_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """C[M,N] = A_e4m3[M,K] @ B_e2m1[N,K]^T; A scales per 1x128, B scales
    ue8m0 per 1x32 (kernel_sm121.py:343-421).  ``b`` is packed two codes per
    byte ``[N, K/2]`` (float4_e2m1fn_x2 or uint8).  Returns bf16 ``[..., N]``."""
    t0 = _time.perf_counter()
    K = a.size(-1)
    M = a.numel() // K
    N = b.size(0)
    out_shape = (*a.shape[:-1], N)
    _require_cuda(a, a_s, b, b_s)
    a_flat = a.view(M, K).contiguous()
    if a_flat.dtype != torch.float8_e4m3fn:
        raise TypeError("fp4_gemm expects a float8_e4m3fn activation")
    b_u8 = b.contiguous().view(torch.uint8)
    if b_u8.shape != (N, K // 2):
        raise ValueError(f"fp4_gemm: weight shape {tuple(b.shape)} does not match K={K}")
    a_sf, as_dt = _scale_arg(a_s.view(M, -1))
    if a_sf.shape != (M, K // 128):
        raise ValueError(f"fp4_gemm: activation scale shape {tuple(a_sf.shape)} does not match M={M}, K={K}")
    if b_s.dtype != torch.float8_e8m0fnu:
        out = _fp4_gemm_fp32_scales(a_flat, a_sf, as_dt, b_u8, b_s, M, N, K)
        _tally("fp4_gemm", t0)
        return out.view(out_shape)
    b_sf = b_s.contiguous()
    if b_sf.shape != (N, K // 32):
        raise ValueError(f"fp4_gemm: scale shapes {tuple(a_sf.shape)} / {tuple(b_sf.shape)} do not match "
                         f"M={M}, N={N}, K={K}")
    out = torch.empty(M, N, device=a.device, dtype=torch.bfloat16)
    _lib.check(_lib.load().bs_fp4_gemm(a_flat.data_ptr(), a_sf.data_ptr(), as_dt, b_u8.data_ptr(),
                                       b_sf.data_ptr(), _lib.DT_E8M0, M, N, K, out.data_ptr(), _stream(a)))
    _tally("fp4_gemm", t0)
    return out.view(out_shape)


def hc_split_sinkhorn(mixes: torch.Tensor, hc_scale: torch.Tensor, hc_base: torch.Tensor, hc_mult: int = 4,
                      sinkhorn_iters: int = 20, eps: float = 1e-6):
    """Hyper-Connection mixing weights (kernel_sm121.py:493-533) in one fused
    kernel.  mixes [b, s, (2+hc)*hc] -> (pre [b,s,hc], post [b,s,hc],
    comb [b,s,hc,hc]), all fp32."""
    t0 = _time.perf_counter()
    _require_cuda(mixes, hc_scale, hc_base)
    b, s, _ = mixes.shape
    hc = hc_mult
    m = mixes.contiguous()
    if m.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        m = m.float()
    n = b * s
    pre = torch.empty(b, s, hc, dtype=torch.float32, device=mixes.device)
    post = torch.empty(b, s, hc, dtype=torch.float32, device=mixes.device)
    comb = torch.empty(b, s, hc, hc, dtype=torch.float32, device=mixes.device)
    sc = hc_scale.float().contiguous()
    bs = hc_base.float().contiguous()
    _lib.check(_lib.load().bs_hc_split_sinkhorn(m.data_ptr(), _X_DT[m.dtype], sc.data_ptr(), bs.data_ptr(), n, hc,
                                                sinkhorn_iters, eps, pre.data_ptr(), post.data_ptr(),
                                                comb.data_ptr(), _stream(mixes)))
    _tally("hc_sinkhorn", t0)
    return pre, post, comb


def sparse_attn(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor, topk_idxs: torch.Tensor,
                softmax_scale: float) -> torch.Tensor:
    """Sparse attention over gathered keys (kernel_sm121.py:430-486).
    q [b, s, h, d], kv [b, n, d], attn_sink [h], topk_idxs [b, s, topk]
    (-1 = no key) -> [b, s, h, d] in q's dtype."""
    t0 = _time.perf_counter()
    _require_cuda(q, kv, attn_sink, topk_idxs)
    b, s, h, d = q.shape
    n = kv.size(1)
    k = topk_idxs.size(-1)
    qc = q.contiguous()
    if qc.dtype not in _X_DT:
        qc = qc.float()
    kvc = kv.contiguous().to(qc.dtype)
    idx = topk_idxs.contiguous()
    if idx.dtype not in (torch.int64, torch.int32):
        idx = idx.long()
    sink = attn_sink.float().contiguous()
    lib = _lib.load()
    out = torch.empty(b, s, h, d, dtype=qc.dtype, device=q.device)
    wsb = lib.bs_sparse_attn_workspace_size(b, s, h, d, k)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=q.device)
    _lib.check(lib.bs_sparse_attn(qc.data_ptr(), kvc.data_ptr(), _X_DT[qc.dtype], sink.data_ptr(), idx.data_ptr(),
                                  1 if idx.dtype == torch.int64 else 0, b, s, h, d, n, k, float(softmax_scale),
                                  out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(q)))
    _tally("sparse_attn", t0)
    return out if out.dtype == q.dtype else out.to(q.dtype)


def indexer_topk(q: torch.Tensor, kv: torch.Tensor, weights: torch.Tensor, topk: int, ratio: int, start_pos: int,
                 offset: int) -> torch.Tensor:
    """The Indexer's score -> top-k step of one rank (kernel_sm121.py:597-642):
    q [1, S, H, D], kv [1, T, D], weights [1, S, H] -> int64 [1, S, topk]
    (key index + offset in descending score order; in prefill, keys at or
    beyond (s+1)//ratio are masked and reported as -1)."""
    t0 = _time.perf_counter()
    _require_cuda(q, kv, weights)
    _, S, H, D = q.shape
    T = kv.size(1)
    qc = q.contiguous()
    if qc.dtype not in _X_DT:
        qc = qc.float()
    kvc = kv.contiguous().to(qc.dtype)
    w = weights.float().contiguous()
    lib = _lib.load()
    out = torch.empty(1, S, topk, dtype=torch.int64, device=q.device)
    ws = torch.empty(max(lib.bs_indexer_topk_workspace_size(S, T), 16), dtype=torch.uint8, device=q.device)
    _lib.check(lib.bs_indexer_topk(qc.data_ptr(), kvc.data_ptr(), _X_DT[qc.dtype], w.data_ptr(), S, H, D, T, topk,
                                   ratio, start_pos, offset, out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(q)))
    _tally("indexer_topk", t0)
    return out
