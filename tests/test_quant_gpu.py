"""CUDA quantisers vs the golden vectors and the oracle: bit for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from gpu_util import bits, cuda_x, np_bits
from oracle import blockscaled as ob

pytestmark = pytest.mark.gpu

DT = {"f32": ob.DT_F32, "e8m0": ob.DT_E8M0, "bf16": ob.DT_BF16}
TDT = {"f32": torch.float32, "e8m0": torch.float8_e8m0fnu}


@pytest.mark.parametrize("name", list(cases.act_quant_inputs().keys()))
@pytest.mark.parametrize("fmt", [None, "ue8m0"])
@pytest.mark.parametrize("sdt", ["f32", "e8m0"])
def test_act_quant_golden(pkg, golden, name, fmt, sdt):
    x, xdt = cases.act_quant_inputs()[name]
    y, s = pkg.act_quant(cuda_x(x, xdt), 128, fmt, TDT[sdt])
    k = f"aq/{name}/{fmt}/{sdt}"
    np.testing.assert_array_equal(bits(y), golden[k + "/y"])
    np.testing.assert_array_equal(bits(s), np_bits(golden[k + "/s"]))
    assert y.shape == x.shape and s.shape == (*x.shape[:-1], x.shape[-1] // 128)


@pytest.mark.parametrize("name", list(cases.act_quant_inputs().keys()))
@pytest.mark.parametrize("fmt", [None, "ue8m0"])
def test_act_quant_inplace_golden(pkg, golden, name, fmt):
    x, xdt = cases.act_quant_inputs()[name]
    t = cuda_x(x, xdt)
    r = pkg.act_quant(t, 128, fmt, torch.float32, True)
    assert r.data_ptr() == t.data_ptr()
    np.testing.assert_array_equal(bits(r), np_bits(golden[f"aq/{name}/{fmt}/inplace"]))


@pytest.mark.parametrize("name", list(cases.fp4_act_quant_inputs().keys()))
def test_fp4_act_quant_golden(pkg, golden, name):
    x, xdt = cases.fp4_act_quant_inputs()[name]
    t = cuda_x(x, xdt)
    r = pkg.fp4_act_quant(t, 32, True)
    np.testing.assert_array_equal(bits(r), np_bits(golden[f"f4q/{name}/out"]))


@pytest.mark.parametrize("block", [32, 64, 128, 256])
@pytest.mark.parametrize("xdt", ["bf16", "f32"])
def test_act_quant_sweep_vs_oracle(pkg, block, xdt):
    """Wide-exponent random inputs, several block sizes, both scale formats."""
    rng = np.random.default_rng(100 + block)
    f = (rng.standard_normal((37, 1024)) * 2.0 ** rng.integers(-20, 20, size=(37, 1))).astype(np.float32)
    x = ob.f32_to_bf16(f) if xdt == "bf16" else f
    for fmt in (None, "ue8m0"):
        y, s = pkg.act_quant(cuda_x(x, xdt), block, fmt, torch.float32)
        ry, rs = ob.act_quant(x, DT[xdt], block, fmt, ob.DT_F32)
        np.testing.assert_array_equal(bits(y), ry)
        np.testing.assert_array_equal(bits(s), np_bits(rs))
    t = cuda_x(x, xdt)
    pkg.fp4_act_quant(t, 32, True)
    np.testing.assert_array_equal(bits(t), np_bits(ob.fp4_act_quant_inplace(x, DT[xdt], 32)))


@pytest.mark.parametrize("sdt", [ob.DT_F32, ob.DT_BF16, ob.DT_F16, ob.DT_E8M0])
@pytest.mark.parametrize("pow2", [0, 1])
def test_act_quant_bf16_128_ragged_all_scale_dtypes(pkg, sdt, pow2):
    """bf16 input with 1x128 blocks through the C ABI: a block count that no
    grid pass divides evenly (plus zero, NaN, inf and tiny blocks), every
    scale dtype, both scale modes."""
    L = pkg._lib
    rng = np.random.default_rng(7 + sdt + 10 * pow2)
    rows, K = 3001, 896  # 21007 blocks
    f = (rng.standard_normal((rows, K)) * 2.0 ** rng.integers(-30, 30, size=(rows, 1))).astype(np.float32)
    f[5, :128] = 0.0
    f[6, 3] = np.nan
    f[7, 200] = np.inf
    f[8, 256:384] = 1e-7
    x = ob.f32_to_bf16(f)
    xt = cuda_x(x, "bf16")
    y = torch.empty(rows, K, device="cuda", dtype=torch.uint8)
    nb = K // 128
    s = torch.empty(rows * nb * (4 if sdt == ob.DT_F32 else 2 if sdt in (ob.DT_BF16, ob.DT_F16) else 1),
                    device="cuda", dtype=torch.uint8)
    L.check(L.load().bs_act_quant(xt.data_ptr(), ob.DT_BF16, rows, K, 128, pow2, y.data_ptr(), s.data_ptr(), sdt,
                                  torch.cuda.current_stream().cuda_stream))
    ry, rs = ob.act_quant(x, ob.DT_BF16, 128, "ue8m0" if pow2 else None, sdt)
    # NaN encodings are the platform's: inf/inf (the inf element over its own
    # inf scale) is +NaN on the GPU (e4m3 0x7F, as the reference's GPU kernel
    # gives) but -NaN from numpy on x86 (0xFF); the NaN block's scale is the
    # canonical NaN on the GPU but keeps the input payload in numpy.  NaNs are
    # therefore compared as NaN, everything else bit for bit.
    def nan_canon(c):
        c = np.array(c, copy=True)
        c[(c & 0x7F) == 0x7F] = 0x7F
        return c
    np.testing.assert_array_equal(nan_canon(bits(y)), nan_canon(ry))
    assert np.count_nonzero(bits(y) != ry) <= 1
    raw = s.cpu().numpy().view(np.asarray(rs).dtype).reshape(rs.shape)
    got, want = ob.to_f32(raw, sdt), ob.to_f32(rs, sdt)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))
    fin = ~np.isnan(want)
    np.testing.assert_array_equal(raw[fin], np.asarray(rs)[fin])


@pytest.mark.parametrize("fmt", [None, "ue8m0"])
def test_act_quant_bf16_every_value_under_many_scales(pkg, fmt):
    """Every finite bf16 magnitude (both signs) quantised under 24 block
    maxima, so x/s meets every e4m3 rounding boundary a bf16 input can reach
    with many non-power-of-two scales.  Each row is [amax, 127 values <= amax]."""
    rng = np.random.default_rng(11)
    codes = np.arange(0, 0x7F80, dtype=np.uint16)  # +0 .. largest finite
    mags = ob.bf16_to_f32(codes)
    amaxes = np.concatenate([[1.0, 3.0, 448.0, 1e-3, 7.5e-5, 1e30],
                             2.0 ** rng.uniform(-20, 40, 18)]).astype(np.float32)
    rows = []
    for A in ob.bf16_to_f32(ob.f32_to_bf16(amaxes)):
        v = codes[mags <= A]
        v = np.where(rng.random(v.shape) < 0.5, v | 0x8000, v).astype(np.uint16)
        n = (len(v) + 126) // 127 * 127
        v = np.concatenate([v, np.zeros(n - len(v), np.uint16)]).reshape(-1, 127)
        rows.append(np.concatenate([np.full((v.shape[0], 1), ob.f32_to_bf16(np.float32(A)), np.uint16), v], axis=1))
    x = np.concatenate(rows)
    y, s = pkg.act_quant(cuda_x(x, "bf16"), 128, fmt, torch.float32)
    ry, rs = ob.act_quant(x, ob.DT_BF16, 128, fmt, ob.DT_F32)
    np.testing.assert_array_equal(bits(y), ry)
    np.testing.assert_array_equal(bits(s), np_bits(rs))


@pytest.mark.parametrize("block", [16, 32, 64, 128])
def test_fp4_act_quant_bf16_every_value(pkg, block):
    """In-place e2m1 fake quantisation of every finite bf16 value (both
    signs) under 24 block maxima, each row [amax, block-1 values <= amax],
    plus blocks holding NaN, inf, zeros and subnormals; the row count leaves
    a ragged last pass."""
    rng = np.random.default_rng(13 + block)
    codes = np.arange(0, 0x7F80, dtype=np.uint16)
    mags = ob.bf16_to_f32(codes)
    amaxes = np.concatenate([[6.0, 1.0, 3e38, 1e-38, 7.0, 0.3],
                             2.0 ** rng.uniform(-120, 120, 18)]).astype(np.float32)
    rows = []
    for A in ob.bf16_to_f32(ob.f32_to_bf16(amaxes)):
        v = codes[mags <= A]
        v = np.where(rng.random(v.shape) < 0.5, v | 0x8000, v).astype(np.uint16)
        n = (len(v) + block - 2) // (block - 1) * (block - 1)
        v = np.concatenate([v, np.zeros(n - len(v), np.uint16)]).reshape(-1, block - 1)
        rows.append(np.concatenate([np.full((v.shape[0], 1), ob.f32_to_bf16(np.float32(A)), np.uint16), v], axis=1))
    x = np.concatenate(rows).reshape(-1)
    special = np.zeros((4, block), np.uint16)
    special[0, 3] = 0x7FC0      # NaN
    special[1, 5] = 0x7F80      # inf
    special[1, 6] = 0x3F80
    special[2, :] = 0x8000      # -0
    special[3, :] = rng.integers(1, 0x80, block) | (rng.integers(0, 2, block) << 15)  # subnormals
    x = np.concatenate([x, special.reshape(-1)])
    K = 4 * block
    x = np.concatenate([x, np.zeros((-len(x)) % K, np.uint16)]).reshape(-1, K)
    t = cuda_x(x, "bf16")
    pkg.fp4_act_quant(t, block, True)
    want = ob.fp4_act_quant_inplace(x, ob.DT_BF16, block)
    got = bits(t)
    nan_g, nan_w = (got & 0x7FFF) > 0x7F80, (want & 0x7FFF) > 0x7F80
    np.testing.assert_array_equal(nan_g, nan_w)  # NaN encodings are the platform's
    np.testing.assert_array_equal(got[~nan_w], want[~nan_w])


def test_act_quant_e4m3_rounding_exhaustive(pkg):
    """Every e4m3 midpoint and its neighbours (ties to even, subnormals)."""
    codes = np.arange(0, 0x7E, dtype=np.uint8)
    v = ob.e4m3_to_f32(codes).astype(np.float64)
    mids = (v[:-1] + v[1:]) / 2
    pts = np.concatenate([v, mids, np.nextafter(mids.astype(np.float32), np.float32(0)),
                          np.nextafter(mids.astype(np.float32), np.float32(1000))]).astype(np.float32)
    pts = np.concatenate([pts, -pts])
    n = (len(pts) + 126) // 127 * 127
    pts = np.concatenate([pts, np.zeros(n - len(pts), np.float32)]).reshape(-1, 127)
    x = np.concatenate([np.full((pts.shape[0], 1), 448.0, np.float32), pts], axis=1)  # scale == 1
    y, s = pkg.act_quant(cuda_x(x, "f32"), 128, None, torch.float32)
    ry, _ = ob.act_quant(x, ob.DT_F32, 128, None, ob.DT_F32)
    np.testing.assert_array_equal(bits(y), ry)


def test_act_quant_leading_dims_and_empty(pkg):
    x = torch.randn(2, 3, 5, 256, device="cuda", dtype=torch.bfloat16)
    y, s = pkg.act_quant(x, 128)
    assert y.shape == x.shape and s.shape == (2, 3, 5, 2)
    e = torch.empty(0, 256, device="cuda", dtype=torch.bfloat16)
    y, s = pkg.act_quant(e, 128)
    assert y.shape == (0, 256) and s.shape == (0, 2)


def test_act_quant_non_contiguous_inplace(pkg):
    base = torch.randn(8, 512, device="cuda", dtype=torch.bfloat16)
    view = base[:, 128:384]
    expect = ob.act_quant_inplace(bits(view.contiguous()), ob.DT_BF16, 128, None)
    pkg.act_quant(view, 128, None, torch.float32, True)
    np.testing.assert_array_equal(bits(base[:, 128:384]), expect)


def test_no_device_error(pkg):
    pkg._lib.device_error_check()
