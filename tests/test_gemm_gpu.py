"""CUDA fp8_gemm / fp4_gemm vs the reference's dequantise-then-matmul result.

Tolerance (from the block-scaled path's spec): relative Frobenius error
<= 1e-2 against the reference / oracle bf16 output; the max-abs error is
printed.  The kernels multiply exact e4m3 x e2m1 products in fp32 and apply
the fp32 block scales per 128-K block, while the reference rounds the
dequantised operands to bf16 first, so ~1e-3 is the expected error.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from conftest import max_abs, rel_fro
from gpu_util import bits, cuda_f32, cuda_u8
from oracle import blockscaled as ob

pytestmark = pytest.mark.gpu

TOL = 1e-2
DT = {"f32": ob.DT_F32, "e8m0": ob.DT_E8M0}


def _scale(a, dt):
    return cuda_f32(a) if dt == "f32" else cuda_u8(a, torch.float8_e8m0fnu)


def run_fp8(pkg, c):
    return pkg.fp8_gemm(cuda_u8(c["a"], torch.float8_e4m3fn), _scale(c["a_s"], c["as_dt"]),
                        cuda_u8(c["b"], torch.float8_e4m3fn), _scale(c["b_s"], c["bs_dt"]))


def run_fp4(pkg, c):
    return pkg.fp4_gemm(cuda_u8(c["a"], torch.float8_e4m3fn), _scale(c["a_s"], c["as_dt"]),
                        cuda_u8(c["b"], torch.float4_e2m1fn_x2), cuda_u8(c["b_s"], torch.float8_e8m0fnu))


def check(out, ref, label):
    e, m = rel_fro(out, ref), max_abs(out, ref)
    print(f"{label}: rel_fro={e:.3e} max_abs={m:.3e}")
    assert e <= TOL, (label, e)
    assert np.isfinite(ob.bf16_to_f32(out)).all(), label


@pytest.mark.parametrize("name", ["small_f32", "small_e8m0", "cfg2"])
def test_fp8_gemm_golden(pkg, golden, name):
    c = cases.fp8_gemm_cases()[name]
    out = bits(run_fp8(pkg, c))
    if out.shape[0] > 1024:
        out = out[::256]
    check(out, golden[f"g8/{name}/out"], f"fp8 {name}")


@pytest.mark.parametrize("name", ["cfg1", "cfg1_ue8m0", "ragged_e8m0", "decode_m1"])
def test_fp4_gemm_golden(pkg, golden, name):
    c = cases.fp4_gemm_cases()[name]
    check(bits(run_fp4(pkg, c)), golden[f"g4/{name}/out"], f"fp4 {name}")


@pytest.mark.parametrize("M", [1, 4, 16, 64])
@pytest.mark.parametrize("N", [2048, 4096])
def test_fp4_decode_sweep(pkg, M, N):
    c = cases.cfg1_fp4(M=M, N=N, K=4096, seed=10 + M + N)
    ref = ob.fp4_gemm(c["a"], c["a_s"], c["b"], c["b_s"], ob.DT_F32, ob.DT_E8M0)
    out = run_fp4(pkg, c)
    check(bits(out), ref, f"fp4 decode M={M} N={N}")
    np.testing.assert_array_equal(bits(run_fp4(pkg, c)), bits(out))  # deterministic


@pytest.mark.parametrize("shape", [(1, 256, 512), (16, 384, 1024), (64, 1024, 4096), (33, 200, 384),
                                   (16, 4096, 2048), (64, 4096, 1024), (32, 7168, 4096)])
def test_fp8_decode_vs_oracle(pkg, shape):
    M, N, K = shape
    rng = np.random.default_rng(M * 7 + N)
    x = ob.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    a, a_s = ob.act_quant(x, ob.DT_BF16, 128, None, ob.DT_F32)
    b, b_s = cases.quant_weight_128x128((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    c = dict(a=a, a_s=a_s, b=b, b_s=b_s, as_dt="f32", bs_dt="f32")
    check(bits(run_fp8(pkg, c)), ob.fp8_gemm(a, a_s, b, b_s), f"fp8 M={M} N={N} K={K}")


@pytest.mark.parametrize("shape", [(256, 512, 1024), (130, 200, 384), (512, 768, 2048)])
def test_fp8_prefill_vs_oracle(pkg, shape):
    M, N, K = shape
    rng = np.random.default_rng(M + N + K)
    x = ob.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    a, a_s = ob.act_quant(x, ob.DT_BF16, 128, None, ob.DT_F32)
    b, b_s = cases.quant_weight_128x128((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    c = dict(a=a, a_s=a_s, b=b, b_s=b_s, as_dt="f32", bs_dt="f32")
    check(bits(run_fp8(pkg, c)), ob.fp8_gemm(a, a_s, b, b_s), f"fp8 M={M} N={N} K={K}")


@pytest.mark.parametrize("shape", [(256, 512, 1024), (130, 200, 384), (300, 1024, 4096)])
@pytest.mark.parametrize("fmt", [None, "ue8m0"])
def test_fp4_prefill_vs_oracle(pkg, shape, fmt):
    M, N, K = shape
    c = cases.cfg1_fp4(M=M, N=N, K=K, scale_fmt=fmt, seed=M + N)
    ref = ob.fp4_gemm(c["a"], c["a_s"], c["b"], c["b_s"], ob.DT_F32, ob.DT_E8M0)
    check(bits(run_fp4(pkg, c)), ref, f"fp4 M={M} N={N} K={K} fmt={fmt}")


def _e8m0_weight_case(rng, N, K):
    """Weights quantised per 128x128 block with power-of-two (ue8m0) scales."""
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    nb, kb = (N + 127) // 128, K // 128
    pad = np.zeros((nb * 128, K), np.float32)
    pad[:N] = w
    blk = pad.reshape(nb, 128, kb, 128)
    amax = np.maximum(np.abs(blk).max(axis=(1, 3)), np.float32(1e-4))
    s = ob.round_scale_pow2((amax / np.float32(448)).astype(np.float32))
    b = ob.f32_to_e4m3(np.clip(blk / s[:, None, :, None], -448, 448).astype(np.float32)).reshape(nb * 128, K)[:N]
    return b, ob.from_f32(s, ob.DT_E8M0)


@pytest.mark.parametrize("shape", [(256, 512, 1024), (130, 200, 384), (512, 768, 2048), (200, 300, 4096)])
def test_fp8_prefill_ue8m0_scales_vs_oracle(pkg, shape):
    """Both scale tensors ue8m0 (the DeepSeek checkpoints' format): the MMA
    applies the scales and accumulates the whole K range in TMEM."""
    M, N, K = shape
    rng = np.random.default_rng(5 * M + N + K)
    x = ob.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    a, a_s = ob.act_quant(x, ob.DT_BF16, 128, "ue8m0", ob.DT_E8M0)
    b, b_s = _e8m0_weight_case(rng, N, K)
    c = dict(a=a, a_s=a_s, b=b, b_s=b_s, as_dt="e8m0", bs_dt="e8m0")
    out = run_fp8(pkg, c)
    check(bits(out), ob.fp8_gemm(a, a_s, b, b_s, ob.DT_E8M0, ob.DT_E8M0), f"fp8 ue8m0 M={M} N={N} K={K}")
    np.testing.assert_array_equal(bits(run_fp8(pkg, c)), bits(out))  # deterministic


@pytest.mark.parametrize("shape", [(256, 512, 1024), (130, 200, 384), (300, 1024, 4096)])
def test_fp4_prefill_ue8m0_act_scales_vs_oracle(pkg, shape):
    """ue8m0 activation scales (act_quant with scale_fmt='ue8m0' and an e8m0
    scale dtype) against the oracle, and against the same scales given as
    fp32."""
    M, N, K = shape
    c = cases.cfg1_fp4(M=M, N=N, K=K, scale_fmt="ue8m0", seed=M + N + 1)
    c = dict(c, a_s=ob.from_f32(c["a_s"], ob.DT_E8M0), as_dt="e8m0")
    ref = ob.fp4_gemm(c["a"], c["a_s"], c["b"], c["b_s"], ob.DT_E8M0, ob.DT_E8M0)
    out = run_fp4(pkg, c)
    check(bits(out), ref, f"fp4 ue8m0 act M={M} N={N} K={K}")
    # the same values as fp32 scales take the promotion path: the two agree closely
    c32 = dict(c, a_s=ob.to_f32(c["a_s"], ob.DT_E8M0), as_dt="f32")
    check(bits(out), bits(run_fp4(pkg, c32)), f"fp4 ue8m0 act vs fp32 scales M={M}")


@pytest.mark.parametrize("shape", [(16, 2048, 4096), (200, 512, 1024), (1, 256, 512)])
@pytest.mark.parametrize("as_dt", ["f32", "e8m0"])
def test_fp4_gemm_fp32_weight_scales_vs_oracle(pkg, shape, as_dt):
    """fp32 weight scales that are not powers of two (kernel_sm121.py:402-406
    multiplies by any fp32 scale): dequantised to bf16 on the device, then
    one bf16 GEMM, as the reference's CPU branch computes it."""
    M, N, K = shape
    c = cases.cfg1_fp4(M=M, N=N, K=K, scale_fmt="ue8m0" if as_dt == "e8m0" else None, seed=M + N + 7)
    if as_dt == "e8m0":
        c = dict(c, a_s=ob.from_f32(c["a_s"], ob.DT_E8M0), as_dt="e8m0")
    rng = np.random.default_rng(N + K)
    b_s32 = (rng.uniform(0.3, 3.0, size=(N, K // 32)) * 2.0 ** rng.integers(-6, 1, size=(N, K // 32))).astype(np.float32)
    ref = ob.fp4_gemm(c["a"], c["a_s"], c["b"], b_s32, DT[c["as_dt"]], ob.DT_F32)
    out = pkg.fp4_gemm(cuda_u8(c["a"], torch.float8_e4m3fn), _scale(c["a_s"], c["as_dt"]),
                       cuda_u8(c["b"], torch.float4_e2m1fn_x2), cuda_f32(b_s32))
    check(bits(out), ref, f"fp4 fp32 weight scales M={M} N={N} K={K} act={as_dt}")


def test_fp8_mx_form_special_scale_bytes(pkg):
    """Both scales ue8m0 (the MX form, scales applied by the MMA).  A block
    whose activation scale byte is 0 contributes 0 in the reference
    (byte << 23 is 0.0) and at most 2^-127 times its products here: the rows
    stay within tolerance.  A byte of 255 is +inf in the reference and NaN in
    the MMA: the affected rows are non-finite in both."""
    M, N, K = 256, 512, 1024
    rng = np.random.default_rng(21)
    x = ob.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    a, a_s = ob.act_quant(x, ob.DT_BF16, 128, "ue8m0", ob.DT_E8M0)
    b, b_s = _e8m0_weight_case(rng, N, K)
    a_s = a_s.copy()
    a_s[3, 2] = 0          # one zero block scale
    a_s[10, :] = 0         # a whole row of zero scales
    ref = ob.fp8_gemm(a, a_s, b, b_s, ob.DT_E8M0, ob.DT_E8M0)
    out = bits(run_fp8(pkg, dict(a=a, a_s=a_s, b=b, b_s=b_s, as_dt="e8m0", bs_dt="e8m0")))
    check(out, ref, "fp8 MX form, zero scale bytes")
    assert np.abs(ob.bf16_to_f32(out[10])).max() < 1e-30
    a_s[20, 1] = 255
    ref = ob.bf16_to_f32(ob.fp8_gemm(a, a_s, b, b_s, ob.DT_E8M0, ob.DT_E8M0))
    out = ob.bf16_to_f32(bits(run_fp8(pkg, dict(a=a, a_s=a_s, b=b, b_s=b_s, as_dt="e8m0", bs_dt="e8m0"))))
    bad_ref, bad_out = ~np.isfinite(ref), ~np.isfinite(out)
    assert bad_ref[20].any() and bad_out[20].all()
    assert not bad_out[np.arange(M) != 20].any() and not bad_ref[np.arange(M) != 20].any()
    np.testing.assert_array_equal(bad_out[20] | ~bad_ref[20], np.ones(N, bool))


def test_gemm_leading_dims(pkg):
    c = cases.cfg1_fp4(M=12, N=256, K=512, seed=3)
    a = cuda_u8(c["a"], torch.float8_e4m3fn).view(3, 4, 512)
    a_s = cuda_f32(c["a_s"]).view(3, 4, 4)
    out = pkg.fp4_gemm(a, a_s, cuda_u8(c["b"], torch.float4_e2m1fn_x2), cuda_u8(c["b_s"], torch.float8_e8m0fnu))
    assert out.shape == (3, 4, 256)
    ref = ob.fp4_gemm(c["a"], c["a_s"], c["b"], c["b_s"], ob.DT_F32, ob.DT_E8M0)
    check(bits(out).reshape(12, 256), ref, "fp4 leading dims")


def test_no_device_error(pkg):
    pkg._lib.device_error_check()


def test_fp8_pair_kernel_parity():
    """The opt-in CTA-pair fp8 kernel (BS_FP8_GEMM_PAIR=1) against the oracle,
    run in a child process so the switch is read fresh."""
    import os
    import subprocess
    import sys
    code = (
        "import sys, numpy as np, torch, importlib; sys.path[:0] = [%r, %r]\n"
        "import cases\nfrom oracle import blockscaled as ob\nfrom conftest import rel_fro\n"
        "from gpu_util import bits, cuda_u8, cuda_f32\n"
        "pkg = importlib.import_module('deepseek-v4-experimental-platform-on-dgx-spark_b200')\n"
        "for (M, N, K) in [(256, 512, 1024), (300, 200, 384), (4096, 4096, 4096)]:\n"
        "    c = cases.cfg2_fp8(M=M, N=N, K=K, seed=M + N)\n"
        "    out = pkg.fp8_gemm(cuda_u8(c['a'], torch.float8_e4m3fn), cuda_f32(c['a_s']),\n"
        "                       cuda_u8(c['b'], torch.float8_e4m3fn), cuda_f32(c['b_s']))\n"
        "    o = bits(out)[::64]; r = ob.fp8_gemm(c['a'], c['a_s'], c['b'], c['b_s'])[::64]\n"
        "    e = rel_fro(o, r); print(M, N, K, e); assert e <= 1e-2\n"
    ) % (os.path.join(os.path.dirname(__file__), "golden"), os.path.dirname(__file__))
    env = dict(os.environ, BS_FP8_GEMM_PAIR="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    print(r.stdout, r.stderr[-2000:])
    assert r.returncode == 0
