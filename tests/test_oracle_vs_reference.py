"""Differential test of the oracle against the reference's own CPU code.

The golden vectors pin the oracle on fixed cases; this test draws fresh
seeded inputs each time (wide exponent ranges, inf / NaN / zero / subnormal
blocks, values a few ulps around rounding ties) and runs them through both
``kernel_sm121`` (its CPU branches, as ``tests/golden/make_golden.py`` does)
and ``oracle.blockscaled``.  It needs the reference project on disk: the
directory comes from the ``BS_REFERENCE_DIR`` environment variable, and the
test skips when it is unset or does not hold ``kernel_sm121.py``.

Quantisers are compared bit for bit, NaNs as NaNs (their sign and payload
are the platform's); GEMMs to 1e-4 relative Frobenius (accumulation order).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

from conftest import rel_fro
from oracle import blockscaled as ob

REF_DIR = os.environ.get("BS_REFERENCE_DIR", "")


@pytest.fixture(scope="module")
def ks():
    if not REF_DIR or not os.path.exists(os.path.join(REF_DIR, "kernel_sm121.py")):
        pytest.skip("BS_REFERENCE_DIR does not point at the reference project")
    sys.path.insert(0, REF_DIR)
    try:
        import kernel_sm121
    finally:
        sys.path.remove(REF_DIR)
    return kernel_sm121


def t_bf16(u16):
    """A bf16 tensor holding a copy of the bits (the in-place modes must not touch the input)."""
    return torch.from_numpy(np.array(u16, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).clone()


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e8m0fnu, torch.uint8):
        return t.view(torch.uint8).numpy()
    return t.numpy().view(np.uint32)


def same_bits_nan_aware(got: np.ndarray, want: np.ndarray, dtype_tag: int):
    g, w = ob.to_f32(got, dtype_tag), ob.to_f32(want, dtype_tag)
    np.testing.assert_array_equal(np.isnan(g), np.isnan(w))
    keep = ~np.isnan(w)
    np.testing.assert_array_equal(np.asarray(got)[keep], np.asarray(want)[keep])


def e4m3_nan_canon(c: np.ndarray) -> np.ndarray:
    c = np.array(c, copy=True)
    c[(c & 0x7F) == 0x7F] = 0x7F
    return c


def random_rows(rng, rows, K, block):
    """bf16 rows: per-row exponent spread, plus special blocks."""
    f = (rng.standard_normal((rows, K)) * 2.0 ** rng.integers(-60, 60, size=(rows, 1))).astype(np.float32)
    f[0, :block] = 0.0
    f[1, 3] = np.nan
    f[2, 5] = np.inf
    f[3, 7] = -np.inf
    f[4, :block] = 2.0 ** -130                          # subnormal block (flushes to the amax floor)
    f[5, :block] = -0.0
    # values straddling e4m3 / e2m1 rounding ties once divided by a power-of-two scale
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 1.0625, 1.1875, 448.0, 464.0], np.float32)
    seg = np.concatenate([ties, np.nextafter(ties, np.float32(0)), np.nextafter(ties, np.float32(1e9))])
    f[6, :seg.size] = seg
    f[6, seg.size] = 448.0
    return ob.f32_to_bf16(f)


@pytest.mark.parametrize("block", [32, 128])
@pytest.mark.parametrize("fmt", [None, "ue8m0"])
@pytest.mark.parametrize("sdt", ["f32", "e8m0"])
def test_act_quant_random_vs_reference(ks, block, fmt, sdt):
    rng = np.random.default_rng(1000 + block + (7 if fmt else 0) + (3 if sdt == "e8m0" else 0))
    x = random_rows(rng, 64, 512, block)
    tdt = torch.float32 if sdt == "f32" else torch.float8_e8m0fnu
    y, s = ks.act_quant(t_bf16(x), block, fmt, tdt, False)
    ry, rs = ob.act_quant(x, ob.DT_BF16, block, fmt, ob.DT_F32 if sdt == "f32" else ob.DT_E8M0)
    np.testing.assert_array_equal(e4m3_nan_canon(bits(y)), e4m3_nan_canon(ry))
    same_bits_nan_aware(bits(s) if sdt == "e8m0" else bits(s).view(np.float32), rs,
                        ob.DT_E8M0 if sdt == "e8m0" else ob.DT_F32)
    r = ks.act_quant(t_bf16(x), block, fmt, torch.float32, True)
    same_bits_nan_aware(bits(r), ob.act_quant_inplace(x, ob.DT_BF16, block, fmt), ob.DT_BF16)


@pytest.mark.parametrize("block", [16, 32, 128])
def test_fp4_act_quant_random_vs_reference(ks, block):
    rng = np.random.default_rng(2000 + block)
    x = random_rows(rng, 64, 512, block)
    r = ks.fp4_act_quant(t_bf16(x), block, True)
    same_bits_nan_aware(bits(r), ob.fp4_act_quant_inplace(x, ob.DT_BF16, block), ob.DT_BF16)


def _e4m3(rng, shape):
    c = rng.integers(0, 256, size=shape, dtype=np.uint8)
    return np.where((c & 0x7F) == 0x7F, c ^ 0x01, c).astype(np.uint8)


@pytest.mark.parametrize("sdt", ["f32", "e8m0"])
def test_fp8_gemm_random_vs_reference(ks, sdt):
    rng = np.random.default_rng(3000 + len(sdt))
    M, N, K = 40, 200, 384
    a, b = _e4m3(rng, (M, K)), _e4m3(rng, (N, K))
    if sdt == "f32":
        a_s = (rng.uniform(0.5, 2.0, (M, K // 128)) * 2.0 ** -6).astype(np.float32)
        b_s = (rng.uniform(0.5, 2.0, ((N + 127) // 128, K // 128)) * 2.0 ** -8).astype(np.float32)
        ta, tb, dt = torch.from_numpy(a_s), torch.from_numpy(b_s), ob.DT_F32
    else:
        a_s = rng.integers(118, 128, (M, K // 128), dtype=np.uint8)
        b_s = rng.integers(118, 128, ((N + 127) // 128, K // 128), dtype=np.uint8)
        ta = torch.from_numpy(a_s).view(torch.float8_e8m0fnu)
        tb = torch.from_numpy(b_s).view(torch.float8_e8m0fnu)
        dt = ob.DT_E8M0
    out = ks.fp8_gemm(torch.from_numpy(a).view(torch.float8_e4m3fn), ta,
                      torch.from_numpy(b).view(torch.float8_e4m3fn), tb)
    ref = ob.fp8_gemm(a, a_s, b, b_s, dt, dt)
    assert rel_fro(bits(out), ref) <= 1e-4


def test_fp4_gemm_random_vs_reference(ks):
    rng = np.random.default_rng(4000)
    M, N, K = 24, 160, 512
    a = _e4m3(rng, (M, K))
    a_s = (rng.uniform(0.5, 2.0, (M, K // 128)) * 2.0 ** -4).astype(np.float32)
    b = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    b_s = (127 - rng.integers(0, 7, (N, K // 32))).astype(np.uint8)
    out = ks.fp4_gemm(torch.from_numpy(a).view(torch.float8_e4m3fn), torch.from_numpy(a_s),
                      torch.from_numpy(b).view(torch.float4_e2m1fn_x2), torch.from_numpy(b_s).view(torch.float8_e8m0fnu))
    ref = ob.fp4_gemm(a, a_s, b, b_s, ob.DT_F32, ob.DT_E8M0)
    assert rel_fro(bits(out), ref) <= 1e-4


@pytest.mark.parametrize("seed,T,E,topk", [(11, 40, 8, 2), (12, 24, 16, 4)])
def test_moe_layer_random_vs_reference(ks, seed, T, E, topk):
    """The MoE oracle against the same composition of the reference's own ops
    (act_quant with ue8m0 scales, fp4_gemm, SiLU in fp32, the top-k weighted
    sum), on fresh seeded cases."""
    import cases
    m = cases.moe_case_small(T=T, H=256, inter=256, E=E, topk=topk, seed=seed)
    x = t_bf16(m["x"])
    idx, w = m["idx"], m["w"]
    inter = m["w13"].shape[1] // 2
    acc = torch.zeros(x.shape, dtype=torch.float32)
    for e in range(E):
        tok, slot = np.nonzero(idx == e)
        if tok.size == 0:
            continue
        h, hs = ks.act_quant(x[torch.from_numpy(tok)], 128, "ue8m0", torch.float32)
        gu = ks.fp4_gemm(h, hs, torch.from_numpy(m["w13"][e]).view(torch.float4_e2m1fn_x2),
                         torch.from_numpy(m["w13_s"][e]).view(torch.float8_e8m0fnu)).float()
        z = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
        q, qs = ks.act_quant(z, 128, "ue8m0", torch.float32)
        y = ks.fp4_gemm(q, qs, torch.from_numpy(m["w2"][e]).view(torch.float4_e2m1fn_x2),
                        torch.from_numpy(m["w2_s"][e]).view(torch.float8_e8m0fnu)).float()
        acc.index_add_(0, torch.from_numpy(tok), torch.from_numpy(w[tok, slot])[:, None] * y)
    got = ob.moe_layer(m["x"], idx, w, m["w13"], m["w13_s"], m["w2"], m["w2_s"])
    assert rel_fro(got, bits(acc.to(torch.bfloat16))) <= 1e-4


@pytest.mark.parametrize("xdt", ["f32", "f16"])
@pytest.mark.parametrize("fmt", [None, "ue8m0"])
def test_quantisers_f32_f16_inputs_vs_reference(ks, xdt, fmt):
    """fp32 and fp16 inputs (the generic kernels' dtypes) through both quantisers."""
    rng = np.random.default_rng(5000 + len(xdt) + (1 if fmt else 0))
    f = ob.bf16_to_f32(random_rows(rng, 48, 256, 128)).astype(np.float32)
    f = f * np.float32(1 + 2.0 ** -9)               # bits below bf16 precision
    if xdt == "f16":
        f = np.clip(f, -60000, 60000)
        x, tag, tt = ob.f32_to_f16(f), ob.DT_F16, torch.from_numpy(ob.f32_to_f16(f).view(np.float16).copy())
    else:
        x, tag, tt = f, ob.DT_F32, torch.from_numpy(f.copy())
    y, s = ks.act_quant(tt.clone(), 128, fmt, torch.float32, False)
    ry, rs = ob.act_quant(x, tag, 128, fmt, ob.DT_F32)
    np.testing.assert_array_equal(e4m3_nan_canon(bits(y)), e4m3_nan_canon(ry))
    same_bits_nan_aware(bits(s).view(np.float32), rs, ob.DT_F32)
    r = ks.fp4_act_quant(tt.clone(), 32, True)
    want = ob.fp4_act_quant_inplace(x, tag, 32)
    got = r.numpy().view(np.uint16) if xdt == "f16" else r.numpy()
    same_bits_nan_aware(got, want, tag)
