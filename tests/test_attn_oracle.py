"""The attention-side oracle (oracle/attn_side.py) against the golden vectors
produced by running the reference's code (tests/golden/make_golden_attn.py).

hc_split_sinkhorn: fp32 results within 4 ulp-scale relative error (the
reference uses torch's vectorised exp / sigmoid, the oracle exact fp64 ones
rounded to fp32); sparse_attn within 1e-5 relative; the Indexer's top-k index
sets equal row by row (orders can differ only between equal scores).
"""

from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import ROOT
from oracle import attn_side as oa

import make_golden_attn as mga


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden_attn.npz"))


def _as_f32(m, dt):
    return (m.astype(np.uint32) << 16).view(np.float32) if dt == "bf16" else m


@pytest.mark.parametrize("name", list(mga.sinkhorn_cases().keys()))
def test_sinkhorn_golden(gold, name):
    m, dt, scale, base, hc, iters, eps = mga.sinkhorn_cases()[name]
    pre, post, comb = oa.hc_split_sinkhorn(_as_f32(m, dt), scale, base, hc, iters, eps)
    for k, v in (("pre", pre), ("post", post), ("comb", comb)):
        g = gold[f"hc/{name}/{k}"]
        assert v.shape == g.shape
        np.testing.assert_allclose(v, g, rtol=5e-6, atol=1e-7, err_msg=f"{name}/{k}")


@pytest.mark.parametrize("name", list(mga.sparse_attn_cases().keys()))
def test_sparse_attn_golden(gold, name):
    q, kv, sink, idx, scale, _ = mga.sparse_attn_cases()[name]
    o = oa.sparse_attn(q, kv, sink, idx, scale)
    np.testing.assert_allclose(o, gold[f"sa/{name}/out"], rtol=1e-5, atol=1e-5)
    assert np.all(o[0, 1] == 0)   # every slot invalid: the sink takes all the weight


@pytest.mark.parametrize("name", list(mga.indexer_cases().keys()))
def test_indexer_topk_golden(gold, name):
    q, kv, w, topk, ratio, start_pos, offset = mga.indexer_cases()[name]
    got = oa.indexer_topk(q, kv, w, topk, ratio, start_pos, offset)
    ref = gold[f"ix/{name}/topk"]
    assert got.shape == ref.shape
    np.testing.assert_array_equal(np.sort(got, axis=-1), np.sort(ref, axis=-1))
