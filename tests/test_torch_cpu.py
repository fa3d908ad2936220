"""The torch restatement of the reference's CPU path (``oracle/torch_cpu.py``,
the reference arm and CPU baseline of ``bench.py``) against the golden
vectors the reference itself produced.

act_quant must match bit for bit; the GEMMs run the same bf16 ``torch.mm`` as
the reference, so they must match to accumulation-order noise (relative
Frobenius < 1e-4); the composed MoE layer within 1e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from conftest import rel_fro
from oracle import torch_cpu as tc


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.view(dtype) if dtype is not None else t


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _scale_t(a, dt):
    return _t(a, torch.float8_e8m0fnu) if dt == "e8m0" else _t(a)


@pytest.mark.parametrize("name", ["cfg1_x", "ragged_bf16", "adv_f32"])
@pytest.mark.parametrize("fmt", [None, "ue8m0"])
def test_act_quant_golden(golden, name, fmt):
    x, xdt = cases.act_quant_inputs()[name]
    xt = _t(x.view(np.int16), torch.bfloat16) if xdt == "bf16" else _t(x)
    y, s = tc.act_quant(xt, 128, pow2=fmt is not None)
    k = f"aq/{name}/{fmt}/f32"
    np.testing.assert_array_equal(y.view(torch.uint8).numpy(), golden[k + "/y"])
    np.testing.assert_array_equal(s.numpy().view(np.uint32), golden[k + "/s"].view(np.uint32))


def test_fp8_gemm_golden(golden):
    for name, c in cases.fp8_gemm_cases().items():
        if name == "cfg2":
            continue  # 4096^3: covered by the oracle's own tests
        o = tc.fp8_gemm(_t(c["a"], torch.float8_e4m3fn), _scale_t(c["a_s"], c["as_dt"]),
                        _t(c["b"], torch.float8_e4m3fn), _scale_t(c["b_s"], c["bs_dt"]))
        assert rel_fro(_bf16_bits(o), golden[f"g8/{name}/out"]) < 1e-4, name


def test_fp4_gemm_golden(golden):
    for name, c in cases.fp4_gemm_cases().items():
        o = tc.fp4_gemm(_t(c["a"], torch.float8_e4m3fn), _scale_t(c["a_s"], c["as_dt"]), _t(c["b"]),
                        _scale_t(c["b_s"], c["bs_dt"]))
        assert rel_fro(_bf16_bits(o), golden[f"g4/{name}/out"]) < 1e-4, name


def test_moe_golden(golden):
    m = cases.moe_case_small()
    x = _t(m["x"].view(np.int16), torch.bfloat16)
    out = torch.zeros(x.shape, dtype=torch.float32)
    E = m["w13"].shape[0]
    tc.moe_experts(x, _t(m["idx"]).long(), _t(m["w"]), range(E), _t(m["w13"]), _t(m["w13_s"], torch.float8_e8m0fnu),
                   _t(m["w2"]), _t(m["w2_s"], torch.float8_e8m0fnu), out)
    assert rel_fro(_bf16_bits(out.to(torch.bfloat16)), golden["moe/small/out"]) < 1e-3
