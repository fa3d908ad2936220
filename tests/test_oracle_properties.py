"""Invariants of the oracle's quantisers (CPU), independent of the golden
vectors: the e4m3 codec round-trips every finite code and rounds to nearest;
act_quant keeps every block inside the e4m3 range with the error of one
rounding; ue8m0 scales are exact powers of two; fp4_act_quant lands on the
e2m1 grid times a power-of-two scale, at the nearest grid point with ties to
the smaller magnitude (kernel_sm121.py:55-124).
"""

from __future__ import annotations

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import blockscaled as ob

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def _bf16(a):
    return ob.f32_to_bf16(np.asarray(a, dtype=np.float32))


def _e4m3_ulp(v):
    """Spacing of e4m3 values around |v| (3 mantissa bits, min normal 2^-6)."""
    e = np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** -6)))
    return np.float32(2.0) ** (e - 3)


def test_e4m3_codes_round_trip():
    codes = np.arange(256, dtype=np.uint8)
    vals = ob.e4m3_to_f32(codes)
    finite = np.isfinite(vals)
    back = ob.f32_to_e4m3(vals[finite])
    # +0 / -0 keep their sign bit; every finite code maps back to itself
    assert np.array_equal(back, codes[finite])
    assert np.nanmax(np.abs(vals)) == 448.0


@settings(max_examples=200, deadline=None)
@given(st.lists(st.floats(-448.0, 448.0, width=32), min_size=1, max_size=64))
def test_e4m3_rounds_to_nearest(xs):
    x = np.array(xs, dtype=np.float32)
    q = ob.e4m3_to_f32(ob.f32_to_e4m3(x))
    assert np.all(np.abs(q - x) <= 0.5 * _e4m3_ulp(x) + 2.0 ** -10)


@pytest.mark.parametrize("pow2", [False, True])
@settings(max_examples=60, deadline=None)
@given(seed=st.integers(0, 2**31 - 1), log_mag=st.floats(-12.0, 12.0))
def test_act_quant_bounds(pow2, seed, log_mag):
    rng = np.random.default_rng(seed)
    x = _bf16(rng.standard_normal((4, 256)).astype(np.float32) * np.float32(2.0 ** log_mag))
    y, s = ob.act_quant(x, ob.DT_BF16, 128, "ue8m0" if pow2 else None)
    q = ob.e4m3_to_f32(y).reshape(4, 2, 128)
    s = np.asarray(s, dtype=np.float32)
    assert np.all(np.isfinite(q)) and np.all(np.abs(q) <= 448.0)
    if pow2:
        m, e = np.frexp(s)
        assert np.all(m == 0.5)                       # exact powers of two
    xf = ob.bf16_to_f32(x).reshape(4, 2, 128)
    amax = np.maximum(np.abs(xf).max(-1), np.float32(1e-4))
    assert np.all(amax / s <= 448.0 * (1 + 2.0 ** -20))
    # one rounding to e4m3 of x/s (itself rounded to fp32): |q - x/s| <= half an
    # e4m3 spacing + the fp32 division's rounding, all in the scaled domain
    t = xf.astype(np.float64) / s[..., None].astype(np.float64)
    assert np.all(np.abs(q - t) <= 0.5 * _e4m3_ulp(t) + np.abs(t) * 2.0 ** -23)


@settings(max_examples=60, deadline=None)
@given(seed=st.integers(0, 2**31 - 1), log_mag=st.floats(-20.0, 20.0))
def test_fp4_act_quant_grid_and_nearest(seed, log_mag):
    rng = np.random.default_rng(seed)
    x = _bf16(rng.standard_normal((2, 64)).astype(np.float32) * np.float32(2.0 ** log_mag))
    out = ob.bf16_to_f32(ob.fp4_act_quant_inplace(x, ob.DT_BF16, 32)).reshape(2, 2, 32)
    xf = ob.bf16_to_f32(x).reshape(2, 2, 32)
    amax = np.maximum(np.abs(xf).max(-1), np.float32(6.0 * 2.0 ** -126))
    s = ob.round_scale_pow2((amax / np.float32(6.0)).astype(np.float32))
    m, _ = np.frexp(s)
    assert np.all(m == 0.5)
    mag = np.abs(out) / s[..., None]
    # every output is a grid point times the block's scale (bf16 holds these exactly here)
    on_grid = np.isclose(mag[..., None], E2M1, rtol=0, atol=0).any(-1)
    assert on_grid.all()
    # nearest grid point to |x|/s, ties to the smaller magnitude
    t = np.minimum(np.abs(xf) / s[..., None], 6.0)
    d = np.abs(t[..., None] - E2M1)
    want = E2M1[np.argmin(d, axis=-1)]
    assert np.array_equal(mag, want)
    assert np.all((np.sign(out) == np.sign(xf)) | (out == 0))
