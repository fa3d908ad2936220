"""CUDA kernels of the attention-side ops against the golden vectors made by
running the reference (tests/golden/make_golden_attn.py) and against the
oracle (oracle/attn_side.py) on larger seeded cases.

Tolerances: fp32 elementwise, relative 2e-5 (+1e-6 absolute) for
hc_split_sinkhorn (CUDA's expf against torch's vectorised exp, a few ulp
through 20 Sinkhorn rounds).
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import ROOT
from gpu_util import cuda_f32
from oracle import attn_side as oa

import make_golden_attn as mga

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden_attn.npz"))


def _mixes(m, dt):
    if dt == "bf16":
        return torch.from_numpy(m.view(np.int16)).view(torch.bfloat16).cuda()
    return cuda_f32(m)


@pytest.mark.parametrize("name", list(mga.sinkhorn_cases().keys()))
def test_hc_sinkhorn_golden(pkg, gold, name):
    m, dt, scale, base, hc, iters, eps = mga.sinkhorn_cases()[name]
    pre, post, comb = pkg.kernel.hc_split_sinkhorn(_mixes(m, dt), cuda_f32(scale), cuda_f32(base), hc, iters, eps)
    for k, v in (("pre", pre), ("post", post), ("comb", comb)):
        g = gold[f"hc/{name}/{k}"]
        got = v.cpu().numpy()
        assert got.shape == g.shape, (k, got.shape, g.shape)
        np.testing.assert_allclose(got, g, rtol=2e-5, atol=1e-6, err_msg=f"{name}/{k}")


@pytest.mark.parametrize("hc,iters,n", [(4, 20, 65536), (4, 20, 1), (2, 7, 1000), (8, 3, 513), (4, 20, 129)])
def test_hc_sinkhorn_vs_oracle(pkg, hc, iters, n):
    rng = np.random.default_rng(hc * 1000 + n)
    m = rng.standard_normal((1, n, (2 + hc) * hc)).astype(np.float32) * 2
    scale = rng.uniform(0.5, 2.0, 3).astype(np.float32)
    base = rng.standard_normal((2 + hc) * hc).astype(np.float32)
    pre, post, comb = pkg.kernel.hc_split_sinkhorn(cuda_f32(m), cuda_f32(scale), cuda_f32(base), hc, iters, 1e-6)
    rp, rq, rc = oa.hc_split_sinkhorn(m, scale, base, hc, iters, 1e-6)
    np.testing.assert_allclose(pre.cpu().numpy(), rp, rtol=2e-5, atol=1e-6)
    np.testing.assert_allclose(post.cpu().numpy(), rq, rtol=2e-5, atol=1e-6)
    np.testing.assert_allclose(comb.cpu().numpy(), rc, rtol=2e-5, atol=1e-6)
    # doubly stochastic after Sinkhorn: columns sum to ~1
    assert np.abs(comb.cpu().numpy().sum(axis=-2) - 1).max() < 1e-3
