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
