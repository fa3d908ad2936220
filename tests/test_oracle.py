"""The oracle against the golden vectors produced by the reference itself (CPU).

Quantisers must match bit for bit; GEMMs must match the reference's bf16
torch.mm output to within accumulation-order noise (rel. Frobenius < 1e-4).
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

import cases
from conftest import rel_fro
from oracle import blockscaled as ob

DT = {"f32": ob.DT_F32, "e8m0": ob.DT_E8M0, "bf16": ob.DT_BF16}


def _bits(a):
    a = np.asarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", list(cases.act_quant_inputs().keys()))
@pytest.mark.parametrize("fmt", [None, "ue8m0"])
@pytest.mark.parametrize("sdt", ["f32", "e8m0"])
def test_act_quant_golden(golden, name, fmt, sdt):
    x, xdt = cases.act_quant_inputs()[name]
    np.testing.assert_array_equal(x, golden[f"aq/{name}/x"])
    y, s = ob.act_quant(x, DT[xdt], 128, fmt, DT[sdt])
    k = f"aq/{name}/{fmt}/{sdt}"
    np.testing.assert_array_equal(y, golden[k + "/y"])
    np.testing.assert_array_equal(_bits(s), _bits(golden[k + "/s"]))


@pytest.mark.parametrize("name", list(cases.act_quant_inputs().keys()))
@pytest.mark.parametrize("fmt", [None, "ue8m0"])
def test_act_quant_inplace_golden(golden, name, fmt):
    x, xdt = cases.act_quant_inputs()[name]
    r = ob.act_quant_inplace(x, DT[xdt], 128, fmt)
    np.testing.assert_array_equal(_bits(r), _bits(golden[f"aq/{name}/{fmt}/inplace"]))


@pytest.mark.parametrize("name", list(cases.fp4_act_quant_inputs().keys()))
def test_fp4_act_quant_golden(golden, name):
    x, xdt = cases.fp4_act_quant_inputs()[name]
    r = ob.fp4_act_quant_inplace(x, DT[xdt], 32)
    np.testing.assert_array_equal(_bits(r), _bits(golden[f"f4q/{name}/out"]))


def test_fp8_gemm_golden(golden):
    for name, c in cases.fp8_gemm_cases().items():
        for k in ("a", "a_s", "b", "b_s"):
            assert _sha(c[k]) == str(golden[f"g8/{name}/sha_{k}"]), (name, k)
        o = ob.fp8_gemm(c["a"], c["a_s"], c["b"], c["b_s"], DT[c["as_dt"]], DT[c["bs_dt"]])
        g = golden[f"g8/{name}/out"]
        if o.shape[0] > 1024:
            o = o[::256]
        assert rel_fro(o, g) < 1e-4, name
        assert (o != g).mean() < 1e-3, name


def test_fp4_gemm_golden(golden):
    for name, c in cases.fp4_gemm_cases().items():
        for k in ("a", "a_s", "b", "b_s"):
            assert _sha(c[k]) == str(golden[f"g4/{name}/sha_{k}"]), (name, k)
        o = ob.fp4_gemm(c["a"], c["a_s"], c["b"], c["b_s"], DT[c["as_dt"]], DT[c["bs_dt"]])
        g = golden[f"g4/{name}/out"]
        assert rel_fro(o, g) < 1e-4, name
        assert (o != g).mean() < 1e-3, name


def test_moe_golden(golden):
    m = cases.moe_case_small()
    assert _sha(m["w13"]) == str(golden["moe/small/sha_w13"])
    o = ob.moe_layer(m["x"], m["idx"], m["w"], m["w13"], m["w13_s"], m["w2"], m["w2_s"])
    assert rel_fro(o, golden["moe/small/out"]) < 1e-3


def test_known_answers():
    # e2m1 table: low nibble = even k, all 16 codes (kernel_sm121.py:263-266)
    b = np.array([[0x10, 0x32, 0x54, 0x76, 0x98, 0xBA, 0xDC, 0xFE]], dtype=np.uint8)
    np.testing.assert_array_equal(ob.dequant_fp4(b)[0], ob.FP4_TABLE)
    # e8m0 decode is a bare exponent placement: 0 -> 0.0, 127 -> 1.0, 255 -> inf
    np.testing.assert_array_equal(ob.e8m0_to_f32(np.array([0, 127, 128, 255], np.uint8)),
                                  np.array([0.0, 1.0, 2.0, np.inf], np.float32))
    # a scale one ulp above a power of two does not round up (fp32 log2)
    assert ob.round_scale_pow2(np.float32(2.0 ** -10) * np.float32(1 + 2.0 ** -23)) == np.float32(2.0 ** -10)
    # special scales follow torch.exp2(torch.ceil(torch.log2(s))): inf -> inf, NaN -> NaN
    import torch
    sp = np.array([np.inf, np.nan, 2.0 ** -130, 1e30, 3.0], np.float32)
    np.testing.assert_array_equal(ob.round_scale_pow2(sp),
                                  torch.exp2(torch.ceil(torch.log2(torch.from_numpy(sp)))).numpy())
    # e4m3 RNE ties go to even; 448 is the largest finite value
    np.testing.assert_array_equal(ob.f32_to_e4m3(np.array([1.0625, 1.1875, 448.0, -448.0], np.float32)),
                                  np.array([0x38, 0x3A, 0x7E, 0xFE], np.uint8))


def test_fp4_act_quant_ties_to_smaller():
    x = np.array([[6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0] + [0.0] * 24], dtype=np.float32)
    r = ob.fp4_act_quant_inplace(x, ob.DT_F32, 32)
    np.testing.assert_array_equal(r[0, :8], np.array([6.0, 0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0], np.float32))
