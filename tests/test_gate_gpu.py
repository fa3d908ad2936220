"""Gate projection on the tensor cores (bs_moe_gate / moe.gate_logits) and the
gated MoE layer.

logits = x . Wg^T with bf16 operands and fp32 accumulation: compared with an
fp64 product of the same bf16 values, relative error <= 1e-5 per row norm.
The gated layer (gate weight in, no host round trip) equals the layer given
those logits bit for bit, and the oracle composition on small shapes within
the MoE tolerance (relative Frobenius 1e-2).
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

import cases
from conftest import PKG_NAME, rel_fro
from gpu_util import bits, cuda_u8
from oracle import blockscaled as ob

pytestmark = pytest.mark.gpu


def moe_mod():
    return importlib.import_module(PKG_NAME + ".moe")


@pytest.mark.parametrize("T,H,E", [(1024, 4096, 256), (1, 512, 16), (300, 1024, 64), (129, 256, 384)])
def test_gate_logits_vs_fp64(T, H, E):
    mm = moe_mod()
    g = torch.Generator(device="cuda")
    g.manual_seed(T + E)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(E, H, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    got = mm.gate_logits(x, w).double().cpu()
    ref = x.double().cpu() @ w.double().cpu().T
    err = ((got - ref).norm(dim=1) / ref.norm(dim=1).clamp_min(1e-30)).max().item()
    print(f"gate T={T} H={H} E={E}: max row rel err {err:.2e}")
    assert err <= 1e-5


@pytest.mark.parametrize("T,H,inter,E,topk", [(200, 512, 256, 16, 4), (64, 1024, 512, 32, 8)])
def test_gated_layer(T, H, inter, E, topk):
    mm = moe_mod()
    m = cases.moe_case_small(T=T, H=H, inter=inter, E=E, topk=topk, seed=T + 1)
    W = mm.MoEWeights(cuda_u8(m["w13"]), cuda_u8(m["w13_s"]), cuda_u8(m["w2"]), cuda_u8(m["w2_s"]))
    x = torch.from_numpy(m["x"].view(np.int16)).cuda().view(torch.bfloat16)
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    wg = (torch.randn(E, H, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    gated = mm.moe_forward(x, None, W, topk, gate_weight=wg)
    logits = mm.gate_logits(x, wg)
    given = mm.moe_forward(x, logits, W, topk)
    torch.cuda.synchronize()
    assert torch.equal(gated, given)
    idx, wts = ob.moe_route(logits.cpu().numpy(), topk)
    ref = ob.moe_layer(m["x"], idx, wts, m["w13"], m["w13_s"], m["w2"], m["w2_s"])
    e = rel_fro(bits(gated), ref)
    print(f"gated layer T={T} E={E}: rel_fro={e:.2e}")
    assert e <= 1e-2
