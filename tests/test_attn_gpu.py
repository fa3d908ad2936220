"""CUDA kernels of the attention-side ops against the golden vectors made by
running the reference (tests/golden/make_golden_attn.py) and against the
oracle (oracle/attn_side.py) on larger seeded cases.

Tolerances: fp32 elementwise, relative 2e-5 (+1e-6 absolute) for
hc_split_sinkhorn (CUDA's expf against torch's vectorised exp, a few ulp
through 20 Sinkhorn rounds); sparse_attn relative 1e-4 (fp32 sums of the k
keys in another order); the Indexer's top-k index sets equal row by row.
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


@pytest.mark.parametrize("name", list(mga.sparse_attn_cases().keys()))
def test_sparse_attn_golden(pkg, gold, name):
    q, kv, sink, idx, scale, _ = mga.sparse_attn_cases()[name]
    o = pkg.kernel.sparse_attn(cuda_f32(q), cuda_f32(kv), cuda_f32(sink), torch.from_numpy(idx).cuda(), scale)
    np.testing.assert_allclose(o.cpu().numpy(), gold[f"sa/{name}/out"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("b,s,h,d,n,k", [(1, 3, 16, 576, 300, 256), (2, 1, 8, 128, 5000, 2048),
                                         (1, 400, 4, 64, 128, 64)])
def test_sparse_attn_vs_oracle(pkg, b, s, h, d, n, k):
    """Decode-shaped (keys split across CTAs, merged with the sink) and
    prefill-shaped cases, bf16 inputs, against the oracle on the same values."""
    rng = np.random.default_rng(b * s + h + d)
    q = rng.standard_normal((b, s, h, d)).astype(np.float32)
    kv = rng.standard_normal((b, n, d)).astype(np.float32)
    sink = rng.standard_normal(h).astype(np.float32)
    idx = rng.integers(-1, n, size=(b, s, k)).astype(np.int64)
    qt = torch.from_numpy(q).cuda().to(torch.bfloat16)
    kvt = torch.from_numpy(kv).cuda().to(torch.bfloat16)
    o = pkg.kernel.sparse_attn(qt, kvt, cuda_f32(sink), torch.from_numpy(idx).cuda(), d ** -0.5)
    assert o.dtype == torch.bfloat16
    ref = oa.sparse_attn(qt.float().cpu().numpy(), kvt.float().cpu().numpy(), sink, idx, d ** -0.5)
    got = o.float().cpu().numpy()
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    print(f"sparse_attn b={b} s={s} h={h} d={d} k={k}: rel_fro={err:.2e}")
    assert err < 5e-3     # bf16 output rounding


@pytest.mark.parametrize("name", list(mga.indexer_cases().keys()))
def test_indexer_topk_golden(pkg, gold, name):
    q, kv, w, topk, ratio, start_pos, offset = mga.indexer_cases()[name]
    got = pkg.kernel.indexer_topk(cuda_f32(q), cuda_f32(kv), cuda_f32(w), topk, ratio, start_pos, offset)
    ref = gold[f"ix/{name}/topk"]
    np.testing.assert_array_equal(np.sort(got.cpu().numpy(), axis=-1), np.sort(ref, axis=-1))


@pytest.mark.parametrize("S,H,D,ratio,topk,start", [(512, 64, 128, 4, 64, 0), (3, 16, 128, 4, 100, 4000),
                                                    (300, 8, 64, 1, 300, 0)])
def test_indexer_topk_vs_oracle(pkg, S, H, D, ratio, topk, start):
    rng = np.random.default_rng(S + H + D)
    T = (start + S) // ratio
    q = rng.standard_normal((1, S, H, D)).astype(np.float32)
    kv = rng.standard_normal((1, T, D)).astype(np.float32)
    w = rng.standard_normal((1, S, H)).astype(np.float32)
    got = pkg.kernel.indexer_topk(cuda_f32(q), cuda_f32(kv), cuda_f32(w), topk, ratio, start, 11).cpu().numpy()
    ref = oa.indexer_topk(q, kv, w, topk, ratio, start, 11)
    np.testing.assert_array_equal(np.sort(got, axis=-1), np.sort(ref, axis=-1))
    # valid picks come in descending score order
    assert (got[0, -1, :min(topk, T)] >= -1).all()
