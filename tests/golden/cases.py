"""Seeded numpy inputs for the golden vectors and the parity tests.

Every generator is deterministic (numpy PCG64 with fixed seeds), so the GPU
tests regenerate exactly the operands the golden file was made from; the
golden file stores a sha256 of each large operand to prove it.
"""

from __future__ import annotations

import os
import sys

import numpy as np

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from oracle import blockscaled as ob  # noqa: E402


def _bf16(a: np.ndarray) -> np.ndarray:
    return ob.f32_to_bf16(np.asarray(a, dtype=np.float32))


def rand_e4m3(rng, shape, sigma=None):
    """Random e4m3 codes without the NaN codes (0x7F, 0xFF)."""
    if sigma is None:
        c = rng.integers(0, 256, size=shape, dtype=np.uint8)
        c = np.where((c & 0x7F) == 0x7F, c ^ 0x01, c).astype(np.uint8)
        return c
    return ob.f32_to_e4m3(np.clip(rng.normal(0, sigma, size=shape), -448, 448).astype(np.float32))


def act_quant_inputs():
    rng = np.random.default_rng(0)
    cases = {}
    cases["cfg1_x"] = (_bf16(rng.standard_normal((16, 4096))), "bf16")
    mag = 10.0 ** rng.uniform(-6, 3, size=(3, 5, 1))
    cases["ragged_bf16"] = (_bf16(rng.standard_normal((3, 5, 256)) * mag), "bf16")

    adv = np.zeros((8, 512), dtype=np.float32)
    # row 0: all zeros -> amax floor 1e-4
    # row 1: block scales a few ulp above a power of two
    for blk, k in enumerate([1, 2, 3, 40]):
        v = np.float32(448.0 * 2.0 ** -10) * np.float32(1 + k * 2.0 ** -23)
        adv[1, blk * 128:(blk + 1) * 128] = rng.uniform(-1, 1, 128).astype(np.float32) * v
        adv[1, blk * 128] = v
    # row 2: e4m3 rounding ties at scale 1 (amax = 448)
    ties = []
    for e in range(-9, 9):
        for m in range(8):
            lo = (1 + m / 8) * 2.0 ** e if e >= -6 else m / 8 * 2.0 ** -6
            step = 2.0 ** (e - 3) if e >= -6 else 2.0 ** -9
            ties.append(lo + step / 2)
    ties = np.array(ties[:127], dtype=np.float32)
    for blk in range(4):
        adv[2, blk * 128] = 448.0
        adv[2, blk * 128 + 1:blk * 128 + 128] = ties * (1 if blk % 2 == 0 else -1)
    # row 3: signed zeros and fp32 subnormals
    adv[3, :] = -0.0
    adv[3, 128:256] = (rng.uniform(-1, 1, 128) * 1e-39).astype(np.float32)
    adv[3, 300] = 1e-3
    # row 4: very large values
    adv[4, :] = (rng.standard_normal(512) * 1e30).astype(np.float32)
    # row 5: one large value per block, the rest underflows
    adv[5, :] = (rng.standard_normal(512) * 1e-6).astype(np.float32)
    adv[5, ::128] = 1000.0
    # rows 6-7: wide exponent range
    adv[6:8, :] = (rng.standard_normal((2, 512)) * 2.0 ** rng.integers(-30, 30, size=(2, 512))).astype(np.float32)
    cases["adv_f32"] = (adv, "f32")
    return cases


def fp4_act_quant_inputs():
    rng = np.random.default_rng(1)
    cases = {}
    cases["rand_bf16"] = (_bf16(rng.standard_normal((4, 2, 128)) * 3.0), "bf16")
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0,
                     0.2, 0.3, 0.7, 0.8, 1.2, 1.3, 1.7, 1.8, 2.4, 2.6, 3.4, 3.6, 4.9, 5.1,
                     0.0, -0.0, 7.0, 5.99], dtype=np.float32)
    t = np.zeros((4, 64), dtype=np.float32)
    for r in range(4):
        blk = np.concatenate([[6.0], ties]).astype(np.float32)
        t[r, :32] = blk * (1 if r % 2 == 0 else -1) * 2.0 ** (r - 1)
        t[r, 32:] = -blk[::-1] * 2.0 ** (r + 3)
    cases["ties_f32"] = (t, "f32")
    cases["tiny_bf16"] = (_bf16(rng.standard_normal((2, 64)) * 1e-38), "bf16")
    return cases


def _weights_fp4(rng, n, k):
    b = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    b_s = (127 + rng.integers(-6, 1, size=(n, k // 32))).astype(np.uint8)
    return b, b_s


def fp8_gemm_cases():
    cases = {}
    rng = np.random.default_rng(2)
    M, N, K = 48, 320, 512
    a = rand_e4m3(rng, (M, K))
    b = rand_e4m3(rng, (N, K))
    a_s = (rng.uniform(0.5, 2.0, (M, K // 128)) * 2.0 ** rng.integers(-8, 1, (M, K // 128))).astype(np.float32)
    b_s = (rng.uniform(0.5, 2.0, ((N + 127) // 128, K // 128)) * 2.0 ** -8).astype(np.float32)
    cases["small_f32"] = dict(a=a, a_s=a_s, b=b, b_s=b_s, as_dt="f32", bs_dt="f32")
    a_s8 = rng.integers(118, 128, (M, K // 128), dtype=np.uint8)
    b_s8 = rng.integers(118, 128, ((N + 127) // 128, K // 128), dtype=np.uint8)
    cases["small_e8m0"] = dict(a=a, a_s=a_s8, b=b, b_s=b_s8, as_dt="e8m0", bs_dt="e8m0")
    cases["cfg2"] = cfg2_fp8()
    return cases


def cfg2_fp8(M=4096, N=4096, K=4096, seed=3):
    """Dense prefill fp8 GEMM operands: A = act_quant(N(0,1)), W = N(0,0.02) per-128x128."""
    rng = np.random.default_rng(seed)
    x = _bf16(rng.standard_normal((M, K), dtype=np.float32))
    a, a_s = ob.act_quant(x, ob.DT_BF16, 128, None, ob.DT_F32)
    w = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    b, b_s = quant_weight_128x128(w)
    return dict(a=a, a_s=a_s, b=b, b_s=b_s, as_dt="f32", bs_dt="f32")


def quant_weight_128x128(w: np.ndarray):
    """Per 128x128 block: s = max(amax,1e-4)/448; e4m3(clamp(w/s, +-448))."""
    N, K = w.shape
    nb, kb = (N + 127) // 128, K // 128
    pad = np.zeros((nb * 128, K), dtype=np.float32)
    pad[:N] = w
    blk = pad.reshape(nb, 128, kb, 128)
    amax = np.abs(blk).max(axis=(1, 3))
    if N % 128:
        amax[-1] = np.abs(w[(nb - 1) * 128:].reshape(N - (nb - 1) * 128, kb, 128)).max(axis=(0, 2))
    s = (np.maximum(amax, np.float32(1e-4)) / np.float32(448)).astype(np.float32)
    q = np.clip(blk / s[:, None, :, None], -448, 448).astype(np.float32)
    b = ob.f32_to_e4m3(q).reshape(nb * 128, K)[:N]
    return b, s


def fp4_gemm_cases():
    cases = {}
    cases["cfg1"] = cfg1_fp4(scale_fmt=None)
    cases["cfg1_ue8m0"] = cfg1_fp4(scale_fmt="ue8m0")
    rng = np.random.default_rng(5)
    M, N, K = 5, 256, 256
    a = rand_e4m3(rng, (M, K), sigma=30.0)
    a_s = rng.integers(118, 128, (M, K // 128), dtype=np.uint8)
    b, b_s = _weights_fp4(rng, N, K)
    cases["ragged_e8m0"] = dict(a=a, a_s=a_s, b=b, b_s=b_s, as_dt="e8m0", bs_dt="e8m0")
    rng = np.random.default_rng(6)
    x = _bf16(rng.standard_normal((1, 4096), dtype=np.float32))
    a, a_s = ob.act_quant(x, ob.DT_BF16, 128, None, ob.DT_F32)
    b, b_s = _weights_fp4(rng, 4096, 4096)
    cases["decode_m1"] = dict(a=a, a_s=a_s, b=b, b_s=b_s, as_dt="f32", bs_dt="e8m0")
    return cases


def cfg1_fp4(M=16, N=2048, K=4096, scale_fmt=None, seed=4):
    """Config-1 operands: A = act_quant(N(0,1) bf16), B uniform e2m1 codes, scales 2^U{-6..0}."""
    rng = np.random.default_rng(seed)
    x = _bf16(rng.standard_normal((M, K), dtype=np.float32))
    a, a_s = ob.act_quant(x, ob.DT_BF16, 128, scale_fmt, ob.DT_F32)
    b, b_s = _weights_fp4(rng, N, K)
    return dict(a=a, a_s=a_s, b=b, b_s=b_s, as_dt="f32", bs_dt="e8m0")


def moe_case_small(T=32, H=256, inter=128, E=8, topk=2, seed=7):
    rng = np.random.default_rng(seed)
    x = _bf16(rng.standard_normal((T, H), dtype=np.float32))
    logits = rng.standard_normal((T, E), dtype=np.float32)
    idx, w = ob.moe_route(logits, topk)
    w13, w13_s = _weights_fp4(rng, E * 2 * inter, H)
    w2, w2_s = _weights_fp4(rng, E * H, inter)
    return dict(x=x, logits=logits, idx=idx, w=w,
                w13=w13.reshape(E, 2 * inter, H // 2), w13_s=w13_s.reshape(E, 2 * inter, H // 32),
                w2=w2.reshape(E, H, inter // 2), w2_s=w2_s.reshape(E, H, inter // 32))
