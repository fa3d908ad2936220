"""numpy restatement of the reference's block-scaled quantise / GEMM CPU path.

Test infrastructure only (see the package docstring).  Every tensor crosses
this module as raw bits in numpy integer arrays so that rounding is explicit:

  * bf16  -> ``np.uint16`` bit patterns
  * e4m3  -> ``np.uint8`` (float8_e4m3fn codes)
  * e8m0  -> ``np.uint8`` (float8_e8m0fnu codes)
  * e2m1x2 -> ``np.uint8``, two codes per byte (low nibble = even k)
  * fp32  -> ``np.float32``

Reference citations are to ``kernel_sm121.py`` of the reference project.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "DT_F32", "DT_BF16", "DT_F16", "DT_E4M3", "DT_E8M0",
    "bf16_to_f32", "f32_to_bf16", "f16_to_f32", "f32_to_f16",
    "e4m3_to_f32", "f32_to_e4m3", "e8m0_to_f32", "f32_to_e8m0",
    "ceil_log2_f32", "round_scale_pow2",
    "act_quant", "act_quant_inplace", "fp4_act_quant_inplace",
    "dequant_fp4", "FP4_TABLE", "fp8_gemm", "fp4_gemm",
    "to_f32", "from_f32", "moe_route", "moe_layer", "silu_f32",
]

# dtype tags shared with the C-ABI (include/bsgemm.h: bs_dtype)
DT_F32, DT_BF16, DT_F16, DT_E4M3, DT_E8M0 = 0, 1, 2, 3, 4

# ---------------------------------------------------------------------------
# scalar formats
# ---------------------------------------------------------------------------


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round-to-nearest-even; NaN -> 0x7FC0 (c10 rule)."""
    f = np.asarray(f, dtype=np.float32)
    bits = f.view(np.uint32)
    # bits + 0x7FFF + lsb stays below 2^32 for every non-NaN pattern (the
    # largest, -inf 0xFF800000, gains at most 0x8000), and NaNs are replaced
    acc = (bits >> 16) & np.uint32(1)
    acc += np.uint32(0x7FFF)
    with np.errstate(over="ignore"):
        acc += bits
    acc >>= 16
    return np.where(np.isnan(f), np.uint16(0x7FC0), acc.astype(np.uint16)).astype(np.uint16)


def f16_to_f32(u16: np.ndarray) -> np.ndarray:
    return np.asarray(u16, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_f16(f: np.ndarray) -> np.ndarray:
    """Round to nearest even; beyond the fp16 range gives inf, as torch's cast does."""
    with np.errstate(over="ignore"):
        return np.asarray(f, dtype=np.float32).astype(np.float16).view(np.uint16)


def _e4m3_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for c in range(256):
        s = -1.0 if c & 0x80 else 1.0
        e = (c >> 3) & 0xF
        m = c & 0x7
        if e == 0xF and m == 0x7:
            t[c] = np.nan
        elif e == 0:
            t[c] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[c] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


_E4M3_TABLE = _e4m3_table()


def e4m3_to_f32(u8: np.ndarray) -> np.ndarray:
    return _E4M3_TABLE[np.asarray(u8, dtype=np.uint8)]


def f32_to_e4m3(f: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn code, RNE, |x| >= 480 -> NaN code (0x7F|sign).

    Same arithmetic as torch's c10 ``fp8e4m3fn_from_fp32_value`` (which the
    reference reaches through ``Tensor.to(torch.float8_e4m3fn)``,
    kernel_sm121.py:83): normal numbers round by a bias trick on the bits,
    numbers below 2^-6 round through an fp32 add of 2^14.
    """
    f = np.asarray(f, dtype=np.float32)
    bits = f.view(np.uint32).astype(np.uint64)
    sign = bits & 0x80000000
    mag = bits ^ sign
    fp8_max = np.uint64(1087 << 20)
    denorm_mask = np.uint64(141 << 23)
    # subnormal branch: fp32 add with 2^14 rounds at the 2^-9 quantum (RNE)
    magf = mag.astype(np.uint32).view(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        sub = (magf + np.float32(2.0 ** 14)).view(np.uint32).astype(np.uint64) - denorm_mask
    mant_odd = (mag >> 20) & 1
    nrm = (mag + np.uint64(((7 - 127) << 23) & 0xFFFFFFFF) + 0x7FFFF + mant_odd) & 0xFFFFFFFF
    nrm = nrm >> 20
    res = np.where(mag >= fp8_max, 0x7F, np.where(mag < np.uint64(121 << 23), sub, nrm))
    res = (res & 0xFF) | (sign >> 24)
    return res.astype(np.uint8)


def e8m0_to_f32(u8: np.ndarray) -> np.ndarray:
    """The reference's e8m0 decode: ``(u8 << 23).view(float32)``.

    kernel_sm121.py:131-133.  Code 0 decodes to 0.0 (not 2^-127) and code 255
    decodes to +inf, because the byte is placed straight into the exponent.
    """
    return (np.asarray(u8, dtype=np.uint8).astype(np.uint32) << 23).view(np.float32)


def f32_to_e8m0(f: np.ndarray) -> np.ndarray:
    """float32 -> float8_e8m0fnu code as torch rounds it (c10 rule).

    Round-to-nearest-even on the exponent using guard/round/sticky bits of the
    fp32 mantissa; inf/NaN map to 255.  Sign is dropped.
    """
    f = np.asarray(f, dtype=np.float32)
    bits = f.view(np.uint32)
    exp = ((bits >> 23) & 0xFF).astype(np.int32)
    g = (bits & 0x400000) != 0
    r = (bits & 0x200000) != 0
    s = (bits & 0x1FFFFF) != 0
    lsb = exp > 0
    up = g & (r | s | lsb)
    out = np.where(exp == 255, 255, exp + up.astype(np.int32))
    return out.astype(np.uint8)


def ceil_log2_f32(x: np.ndarray) -> np.ndarray:
    """ceil(fp32(log2(x))) for positive normal fp32 x, as an int32.

    torch's fp32 ``log2`` agrees with the correctly rounded log2 on every
    input the quantisers produce (checked against torch on all mantissas
    within 200 ulp above a power of two, exponents -40..19); a float64 log2
    rounded once to fp32 reproduces it.  The rounding matters just above a
    power of two: log2(2^-10 * (1 + 2^-23)) rounds to -10.0 in fp32, so the
    ceiling stays -10 instead of becoming -9.
    """
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        l = np.log2(x.astype(np.float64)).astype(np.float32)
    return np.ceil(l).astype(np.int32)


def round_scale_pow2(scale: np.ndarray) -> np.ndarray:
    """``exp2(ceil(log2(scale)))`` in fp32 (kernel_sm121.py:51-52); NaN stays
    NaN and +inf stays +inf (exp2(ceil(log2(inf))) = inf), as in torch."""
    scale = np.asarray(scale, dtype=np.float32)
    finite = np.isfinite(scale)
    e = ceil_log2_f32(np.where(finite, scale, np.float32(1.0)))
    with np.errstate(over="ignore", invalid="ignore"):
        out = np.ldexp(np.float32(1.0), np.clip(e, -200, 200)).astype(np.float32)
    return np.where(finite, out, scale).astype(np.float32)


def to_f32(x: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == DT_F32:
        return np.asarray(x, dtype=np.float32)
    if dtype == DT_BF16:
        return bf16_to_f32(x)
    if dtype == DT_F16:
        return f16_to_f32(x)
    if dtype == DT_E4M3:
        return e4m3_to_f32(x)
    if dtype == DT_E8M0:
        return e8m0_to_f32(x)
    raise ValueError(f"unknown dtype tag {dtype}")


def from_f32(f: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == DT_F32:
        return np.asarray(f, dtype=np.float32)
    if dtype == DT_BF16:
        return f32_to_bf16(f)
    if dtype == DT_F16:
        return f32_to_f16(f)
    if dtype == DT_E4M3:
        return f32_to_e4m3(f)
    if dtype == DT_E8M0:
        return f32_to_e8m0(f)
    raise ValueError(f"unknown dtype tag {dtype}")


# ---------------------------------------------------------------------------
# quantisers
# ---------------------------------------------------------------------------

_AMAX_FLOOR = np.float32(1e-4)
_E4M3_MAX = np.float32(448.0)


def _act_quant_core(x: np.ndarray, x_dtype: int, block_size: int, pow2: bool):
    z = to_f32(x, x_dtype)
    K = z.shape[-1]
    assert K % block_size == 0
    flat = z.reshape(-1, K)
    blocks = flat.reshape(flat.shape[0], K // block_size, block_size)
    with np.errstate(invalid="ignore"):
        amax = np.max(np.abs(blocks), axis=-1)
        amax = np.maximum(amax, _AMAX_FLOOR)  # NaN propagates like torch.clamp
        scale = (amax / _E4M3_MAX).astype(np.float32)
        if pow2:
            scale = round_scale_pow2(scale)
        scaled = (blocks / scale[..., None]).astype(np.float32)
        clamped = np.clip(scaled, -_E4M3_MAX, _E4M3_MAX)
    return flat.shape, blocks.shape, scale, clamped


def act_quant(x: np.ndarray, x_dtype: int = DT_BF16, block_size: int = 128,
              scale_fmt=None, scale_dtype: int = DT_F32):
    """Block-wise e4m3 quantisation, kernel_sm121.py:55-87 (non-inplace branch).

    Per 1 x block_size block of the last dim: amax = max|x| clamped to
    >= 1e-4; scale = amax/448 (``_round_scale_pow2`` when scale_fmt is set);
    y = e4m3(clamp(x/scale, +-448)).  Returns (y codes shaped like x,
    scales shaped [..., K/block_size] in ``scale_dtype``).
    """
    shape = np.shape(x)
    K = shape[-1]
    _, _, scale, clamped = _act_quant_core(x, x_dtype, block_size, scale_fmt is not None)
    y = f32_to_e4m3(clamped).reshape(shape)
    s = from_f32(scale, scale_dtype).reshape(*shape[:-1], K // block_size)
    return y, s


def act_quant_inplace(x: np.ndarray, x_dtype: int = DT_BF16, block_size: int = 128,
                      scale_fmt=None) -> np.ndarray:
    """Quantise-dequantise back to x's dtype, kernel_sm121.py:75-81."""
    shape = np.shape(x)
    _, _, scale, clamped = _act_quant_core(x, x_dtype, block_size, scale_fmt is not None)
    with np.errstate(invalid="ignore", over="ignore"):   # NaN / inf blocks stay NaN / inf
        q = (e4m3_to_f32(f32_to_e4m3(clamped)) * scale[..., None]).astype(np.float32)
    return from_f32(q.reshape(shape), x_dtype)


_FP4_MAX = np.float32(6.0)
_FP4_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def fp4_act_quant_inplace(x: np.ndarray, x_dtype: int = DT_BF16, block_size: int = 32) -> np.ndarray:
    """e2m1 fake quantisation, kernel_sm121.py:94-121 (inplace branch).

    scale = 2^ceil(log2(max(amax, 6*2^-126)/6)); each |x/scale| (clamped to
    6) goes to the nearest of {0,.5,1,1.5,2,3,4,6} with ties to the smaller
    magnitude (``argmin`` keeps the first index); the sign comes from
    ``torch.sign`` (which gives +0 for -0 and for NaN); the product is cast
    back to x's dtype.
    """
    shape = np.shape(x)
    z = to_f32(x, x_dtype)
    K = shape[-1]
    assert K % block_size == 0
    blocks = z.reshape(-1, K // block_size, block_size)
    with np.errstate(invalid="ignore"):
        amax = np.maximum(np.max(np.abs(blocks), axis=-1), np.float32(6.0 * 2.0 ** -126))
        scale = round_scale_pow2((amax / _FP4_MAX).astype(np.float32))
        scaled = (blocks / scale[..., None]).astype(np.float32)
        clamped = np.clip(scaled, -_FP4_MAX, _FP4_MAX)
        signs = np.where(clamped > 0, np.float32(1), np.where(clamped < 0, np.float32(-1), np.float32(0)))
        diffs = np.abs(np.abs(clamped)[..., None] - _FP4_VALUES)
        idx = np.argmin(diffs, axis=-1)
        quant = (signs * _FP4_VALUES[idx]).astype(np.float32)
        res = (quant * scale[..., None]).astype(np.float32)
    return from_f32(res.reshape(shape), x_dtype)


# ---------------------------------------------------------------------------
# GEMMs: dequantise -> bf16 -> matmul, exactly the reference CPU branches
# ---------------------------------------------------------------------------

FP4_TABLE = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                      0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


# every byte's two decoded values: [byte] -> (low nibble, high nibble)
_FP4_PAIRS = np.stack([FP4_TABLE[np.arange(256) & 0x0F], FP4_TABLE[np.arange(256) >> 4]], axis=-1)


def dequant_fp4(b: np.ndarray) -> np.ndarray:
    """Packed e2m1 [N, K/2] -> fp32 [N, K] (kernel_sm121.py:263-266, 334-340).

    Low nibble holds the even k, high nibble the odd k.
    """
    b = np.asarray(b, dtype=np.uint8)
    return _FP4_PAIRS[b].reshape(*b.shape[:-1], b.shape[-1] * 2)


def _scales_f32(s: np.ndarray, dtype: int) -> np.ndarray:
    return to_f32(s, dtype).astype(np.float32)


def _mm_bf16(a_deq_bf16: np.ndarray, b_deq_bf16: np.ndarray) -> np.ndarray:
    """bf16 x bf16^T matmul with fp32 accumulation (as torch.mm's CPU bf16
    kernel does), rounded to bf16."""
    a = bf16_to_f32(a_deq_bf16)
    b = bf16_to_f32(b_deq_bf16)
    return f32_to_bf16(np.matmul(a, b.T, dtype=np.float32))


def fp8_gemm(a: np.ndarray, a_s: np.ndarray, b: np.ndarray, b_s: np.ndarray,
             as_dtype: int = DT_F32, bs_dtype: int = DT_F32) -> np.ndarray:
    """C = A_e4m3 @ B_e4m3^T with 1x128 (A) and 128x128 (B) block scales.

    CPU branch of kernel_sm121.py:236-251: A is dequantised per 1x128 block
    and rounded to bf16; B is dequantised per 128-row block (the last block
    may be ragged) and rounded to bf16; then one bf16 matmul.
    Returns bf16 bits shaped [..., N].
    """
    K = a.shape[-1]
    M = int(np.prod(a.shape[:-1])) if a.ndim > 1 else 1
    N = b.shape[0]
    nk = K // 128
    a_f = e4m3_to_f32(a.reshape(M, K)).reshape(M, nk, 128)
    a_sf = _scales_f32(a_s, as_dtype).reshape(M, nk)
    a_deq = f32_to_bf16((a_f * a_sf[..., None]).astype(np.float32).reshape(M, K))
    b_f = e4m3_to_f32(b).reshape(N, K)
    b_sf = _scales_f32(b_s, bs_dtype)
    nbn = b_sf.shape[0]
    b_deq = np.empty((N, K), dtype=np.float32)
    for i in range(nbn):
        st, en = i * 128, min(i * 128 + 128, N)
        rows = b_f[st:en].reshape(en - st, nk, 128) * b_sf[i][None, :, None]
        b_deq[st:en] = rows.reshape(en - st, K)
    out = _mm_bf16(a_deq, f32_to_bf16(b_deq))
    return out.reshape(*a.shape[:-1], N)


def fp4_gemm(a: np.ndarray, a_s: np.ndarray, b: np.ndarray, b_s: np.ndarray,
             as_dtype: int = DT_F32, bs_dtype: int = DT_E8M0) -> np.ndarray:
    """C = A_e4m3 @ B_e2m1^T; A scales per 1x128, B scales per 1x32.

    CPU branch of kernel_sm121.py:395-417: B is LUT-dequantised, multiplied
    by its per-32 scales and rounded to bf16; A is dequantised per 128 and
    rounded to bf16; then one bf16 matmul.  Returns bf16 bits [..., N].
    """
    K = a.shape[-1]
    M = int(np.prod(a.shape[:-1])) if a.ndim > 1 else 1
    N = b.shape[0]
    b_sf = _scales_f32(b_s, bs_dtype).reshape(N, K // 32)
    b_deq = (dequant_fp4(b).reshape(N, K // 32, 32) * b_sf[..., None]).astype(np.float32)
    b_deq = f32_to_bf16(b_deq.reshape(N, K))
    a_sf = _scales_f32(a_s, as_dtype).reshape(M, K // 128)
    a_deq = (e4m3_to_f32(a.reshape(M, K)).reshape(M, K // 128, 128) * a_sf[..., None]).astype(np.float32)
    a_deq = f32_to_bf16(a_deq.reshape(M, K))
    out = _mm_bf16(a_deq, b_deq)
    return out.reshape(*a.shape[:-1], N)


# ---------------------------------------------------------------------------
# composed MoE layer (the reference's caller lives in the unvendored model.py)
# ---------------------------------------------------------------------------


def silu_f32(g: np.ndarray) -> np.ndarray:
    g = np.asarray(g, dtype=np.float32)
    with np.errstate(over="ignore"):
        return (g / (np.float32(1.0) + np.exp(-g.astype(np.float64)).astype(np.float32))).astype(np.float32)


def moe_route(logits: np.ndarray, topk: int):
    """Top-k expert choice and softmax-over-top-k weights (fp32).

    The selection keeps the k largest logits per token (ties: lower expert
    index first); weights = softmax of those k logits.
    """
    logits = np.asarray(logits, dtype=np.float32)
    order = np.argsort(-logits, axis=-1, kind="stable")[:, :topk]
    top = np.take_along_axis(logits, order, axis=-1).astype(np.float64)
    w = np.exp(top - top.max(axis=-1, keepdims=True))
    w = (w / w.sum(axis=-1, keepdims=True)).astype(np.float32)
    return order.astype(np.int32), w


def moe_layer(x_bf16: np.ndarray, idx: np.ndarray, w: np.ndarray,
              w13: np.ndarray, w13_s: np.ndarray, w2: np.ndarray, w2_s: np.ndarray,
              experts=None, workers: int = 1) -> np.ndarray:
    """MoE layer composed from the reference ops, expert by expert.

    Per expert e and its routed tokens: h = act_quant(x, 128, "ue8m0");
    g = fp4_gemm(h, W1_e), u = fp4_gemm(h, W3_e) (bf16 outputs; W13_e holds
    W1_e in rows [0, I) and W3_e in rows [I, 2I)); z = silu(g) * u in fp32;
    q = act_quant(z, 128, "ue8m0"); y = fp4_gemm(q, W2_e); the token output
    is sum_k w[t,k] * y_k accumulated in fp32, rounded to bf16.
    ``experts`` restricts the computation to a subset (contributions from
    other experts are left out), for sampled checks at large sizes.  The
    weight arguments only need ``.shape`` and ``[e]`` (so a caller can fetch
    one expert at a time); ``workers`` > 1 computes the experts' outputs on
    that many threads and still sums them in expert order (same result).
    """
    T, H = x_bf16.shape
    E, twoI, _ = w13.shape
    inter = twoI // 2
    out = np.zeros((T, H), dtype=np.float32)
    ex_list = range(E) if experts is None else experts

    def expert(e):
        tok, slot = np.nonzero(idx == e)
        if tok.size == 0:
            return None
        h, hs = act_quant(x_bf16[tok], DT_BF16, 128, "ue8m0", DT_F32)
        gu = bf16_to_f32(fp4_gemm(h, hs, w13[e], w13_s[e], DT_F32, DT_E8M0))
        z = (silu_f32(gu[:, :inter]) * gu[:, inter:]).astype(np.float32)
        q, qs = act_quant(z, DT_F32, 128, "ue8m0", DT_F32)
        y = bf16_to_f32(fp4_gemm(q, qs, w2[e], w2_s[e], DT_F32, DT_E8M0))
        return tok, slot, y

    if workers > 1:
        from concurrent.futures import ThreadPoolExecutor
        with ThreadPoolExecutor(workers) as pool:
            parts = list(pool.map(expert, ex_list))
    else:
        parts = [expert(e) for e in ex_list]
    for part in parts:
        if part is not None:
            tok, slot, y = part
            np.add.at(out, tok, w[tok, slot][:, None] * y)
    return f32_to_bf16(out)
