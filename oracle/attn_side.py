"""numpy restatement of the reference's attention-side ops that consume the
block-scaled path's outputs.

Test infrastructure only, like ``oracle/blockscaled.py``: it is pinned by the
golden vectors of ``tests/golden/make_golden_attn.py`` (produced by running
the reference) and used as the checker of the CUDA kernels; nothing on the
product path imports it.  Reference citations are to ``kernel_sm121.py``.

All arithmetic is fp32 (the reference promotes to fp32 with ``.float()``);
transcendental functions are evaluated in fp64 and rounded once to fp32.
"""

from __future__ import annotations

import numpy as np

__all__ = ["hc_split_sinkhorn", "sparse_attn", "indexer_topk"]


def _f32(x):
    return np.asarray(x, dtype=np.float32)


def _sigmoid(x):
    x = np.asarray(x, dtype=np.float64)
    with np.errstate(over="ignore"):
        return (1.0 / (1.0 + np.exp(-x))).astype(np.float32)


def hc_split_sinkhorn(mixes, hc_scale, hc_base, hc_mult: int = 4, sinkhorn_iters: int = 20, eps: float = 1e-6):
    """kernel_sm121.py:493-533.  mixes [..., (2+hc)*hc] (fp32 values) ->
    pre [..., hc] = sigmoid(m[:hc]*s0 + b[:hc]) + eps,
    post [..., hc] = 2*sigmoid(m[hc:2hc]*s1 + b[hc:2hc]),
    comb [..., hc, hc]: row softmax of m[2hc:]*s2 + b[2hc:] plus eps, divided by
    its column sums (+eps), then sinkhorn_iters-1 rounds of row then column
    normalisation (each sum + eps)."""
    hc = hc_mult
    m = _f32(mixes)
    lead = m.shape[:-1]
    flat = m.reshape(-1, (2 + hc) * hc)
    s = _f32(hc_scale)
    b = _f32(hc_base)
    e = np.float32(eps)
    pre = _sigmoid(flat[:, :hc] * s[0] + b[:hc]) + e
    post = np.float32(2.0) * _sigmoid(flat[:, hc:2 * hc] * s[1] + b[hc:2 * hc])
    raw = flat[:, 2 * hc:].reshape(-1, hc, hc) * s[2] + b[2 * hc:].reshape(hc, hc)
    mx = raw.max(axis=-1, keepdims=True)
    with np.errstate(over="ignore", invalid="ignore"):
        ex = np.exp((raw - mx).astype(np.float64)).astype(np.float32)
    comb = (ex / ex.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32) + e
    comb = comb / (comb.sum(axis=-2, keepdims=True, dtype=np.float32) + e)
    for _ in range(sinkhorn_iters - 1):
        comb = comb / (comb.sum(axis=-1, keepdims=True, dtype=np.float32) + e)
        comb = comb / (comb.sum(axis=-2, keepdims=True, dtype=np.float32) + e)
    return (pre.reshape(*lead, hc).astype(np.float32), post.reshape(*lead, hc).astype(np.float32),
            comb.reshape(*lead, hc, hc).astype(np.float32))


def sparse_attn(q, kv, attn_sink, topk_idxs, softmax_scale: float):
    """kernel_sm121.py:430-486.  q [b,s,h,d], kv [b,n,d], attn_sink [h],
    topk_idxs [b,s,k] (-1 = no key) -> o [b,s,h,d]: per query, scores
    q . kv[idx] * scale over its k gathered keys (-inf where idx < 0), softmax
    over those k scores and the head's sink logit together, output = the
    k-part of the weights times the gathered keys (the sink takes weight but
    adds no value)."""
    q = _f32(q)
    kv = _f32(kv)
    sink = _f32(attn_sink)
    idx = np.asarray(topk_idxs)
    b, s, h, d = q.shape
    out = np.zeros_like(q)
    for bi in range(b):
        for si in range(s):
            ii = idx[bi, si]
            g = kv[bi, np.clip(ii, 0, None)]                                    # [k, d]
            sc = (q[bi, si].astype(np.float64) @ g.astype(np.float64).T) * softmax_scale   # [h, k]
            sc[:, ii < 0] = -np.inf
            allsc = np.concatenate([sc, sink[:, None].astype(np.float64)], axis=1)
            mx = allsc.max(axis=1, keepdims=True)
            ex = np.exp(allsc - mx)
            wts = ex / ex.sum(axis=1, keepdims=True)
            out[bi, si] = (wts[:, :-1] @ g.astype(np.float64)).astype(np.float32)
    return out


def indexer_topk(q, kv, weights, topk: int, ratio: int, start_pos: int, offset: int):
    """The Indexer's score -> top-k step (kernel_sm121.py:597-642, one rank).
    q [1,S,H,D], kv [1,T,D], weights [1,S,H] -> int64 [1,S,topk]:
    score[s,t] = sum_h relu(q[s,h] . kv[t]) * weights[s,h]; in prefill
    (start_pos == 0) keys t >= (s+1)//ratio are masked to -inf; the topk
    highest-scoring keys (plus offset), masked ones reported as -1.  Rows are
    returned with the valid keys in descending score order."""
    q = _f32(q).astype(np.float64)
    kv = _f32(kv).astype(np.float64)
    w = _f32(weights).astype(np.float64)
    _, S, H, D = q.shape
    T = kv.shape[1]
    out = np.empty((1, S, topk), dtype=np.int64)
    for si in range(S):
        sc = np.maximum(q[0, si] @ kv[0].T, 0.0)                                 # [H, T]
        score = (sc * w[0, si][:, None]).sum(axis=0)
        valid = np.ones(T, bool)
        if start_pos == 0:
            valid = np.arange(T) < (si + 1) // ratio
        score = np.where(valid, score, -np.inf)
        order = np.argsort(-score, kind="stable")[:topk]
        out[0, si] = np.where(valid[order], order + offset, -1)
    return out
