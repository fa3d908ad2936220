"""Golden vectors for the attention-side ops, made by running the reference's own code.

Run once where the reference project is available:

    python tests/golden/make_golden_attn.py <reference project directory>

(or with the directory in ``BS_REFERENCE_DIR``).  It imports ``kernel_sm121``
and calls its CPU code on seeded inputs, writing ``golden_attn.npz`` beside
this file:

  * ``hc_split_sinkhorn`` (kernel_sm121.py:493-533) on mixes of several
    shapes, dtypes, scales and iteration counts, including saturated softmax
    rows, zeros and huge values;
  * ``sparse_attn`` (kernel_sm121.py:430-486) on small q / kv / top-k index
    cases, with invalid (-1) indices, a fully masked query and chunking;
  * the Indexer's score -> top-k step (kernel_sm121.py:597-642, the part of
    ``forward_chunked`` after the projections) written out with the same
    torch operations on given q, kv and head weights, since the method itself
    needs DeepSeek's model module.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def sinkhorn_cases():
    """name -> (mixes, mixes dtype tag, hc_scale, hc_base, hc_mult, iters, eps)"""
    out = {}
    for name, (b, s, hc, iters, dt, sc, seed) in {
        "hc4_b2s33": (2, 33, 4, 20, "f32", 1.0, 1),
        "hc4_b1s300_bf16": (1, 300, 4, 20, "bf16", 1.0, 2),
        "hc4_iters5": (1, 64, 4, 5, "f32", 1.0, 3),
        "hc4_iters1": (1, 17, 4, 1, "f32", 1.0, 4),
        "hc2": (3, 11, 2, 20, "f32", 1.0, 5),
        "hc4_large": (1, 40, 4, 20, "f32", 30.0, 6),
    }.items():
        rng = np.random.default_rng(seed)
        mix = (2 + hc) * hc
        m = (rng.standard_normal((b, s, mix)) * sc).astype(np.float32)
        if name == "hc4_b2s33":
            m[0, 0] = 0.0                    # all-zero row
            m[0, 1, 2 * hc:] = 80.0          # saturated softmax row
            m[1, 2, :hc] = -200.0            # sigmoid underflow
        if dt == "bf16":
            u = m.view(np.uint32)
            m = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        scale = rng.uniform(0.5, 2.0, size=3).astype(np.float32)
        base = rng.standard_normal(mix).astype(np.float32)
        out[name] = (m, dt, scale, base, hc, iters, 1e-6)
    return out


def sparse_attn_cases():
    """name -> (q [b,s,h,d] f32, kv [b,n,d] f32, attn_sink [h], topk_idxs [b,s,k] int64, scale, chunk)"""
    out = {}
    for name, (b, s, h, d, n, k, chunk, seed) in {
        "b1_s5_h4_d32": (1, 5, 4, 32, 20, 8, 512, 11),
        "b2_s7_h3_d64_chunk3": (2, 7, 3, 64, 33, 12, 3, 12),
        "b1_s16_h8_d128": (1, 16, 8, 128, 64, 16, 512, 13),
    }.items():
        rng = np.random.default_rng(seed)
        q = rng.standard_normal((b, s, h, d)).astype(np.float32)
        kv = rng.standard_normal((b, n, d)).astype(np.float32)
        sink = rng.standard_normal(h).astype(np.float32)
        idx = rng.integers(0, n, size=(b, s, k)).astype(np.int64)
        idx[0, 0, k // 2:] = -1              # some invalid slots
        idx[0, 1, :] = -1                    # a query with every slot invalid
        out[name] = (q, kv, sink, idx, float(d) ** -0.5, chunk)
    return out


def indexer_cases():
    """name -> (q [1,S,H,D] f32, kv [1,T,D] f32, weights [1,S,H] f32, topk, ratio, start_pos, offset)"""
    out = {}
    for name, (S, H, D, ratio, topk, start_pos, seed) in {
        "prefill_S40_r4": (40, 4, 32, 4, 6, 0, 21),
        "prefill_S64_r2": (64, 8, 64, 2, 16, 0, 22),
        "decode_pos100": (1, 4, 32, 4, 8, 100, 23),
    }.items():
        rng = np.random.default_rng(seed)
        T = (start_pos + S) // ratio
        q = rng.standard_normal((1, S, H, D)).astype(np.float32)
        kv = rng.standard_normal((1, T, D)).astype(np.float32)
        w = rng.standard_normal((1, S, H)).astype(np.float32)
        out[name] = (q, kv, w, min(topk, T), ratio, start_pos, 7)
    return out


def indexer_reference(q, kv, w, topk, ratio, start_pos, offset, chunk=256):
    """The score -> mask -> top-k steps of kernel_sm121.py:597-642 with the
    same torch operations (one rank: no all-reduce)."""
    _, S, _, _ = q.shape
    T = kv.shape[1]
    out = torch.empty((1, S, topk), dtype=torch.int64)
    arange_T = torch.arange(T)
    seq_arange = torch.arange(1, S + 1)
    for s0 in range(0, S, chunk):
        s1 = min(s0 + chunk, S)
        sc = torch.einsum("bshd,btd->bsht", q[:, s0:s1], kv)
        sc.relu_()
        sc = (sc * w[:, s0:s1].unsqueeze(-1)).sum(dim=2)
        if start_pos == 0:
            thr = seq_arange[s0:s1] // ratio
            sc.masked_fill_((arange_T.unsqueeze(0) >= thr.unsqueeze(1)).unsqueeze(0), float("-inf"))
        top = sc.topk(topk, dim=-1)[1]
        if start_pos == 0:
            thr = seq_arange[s0:s1] // ratio
            invalid = top >= thr.view(1, -1, 1)
            top = top + offset
            top.masked_fill_(invalid, -1)
        else:
            top = top + offset
        out[:, s0:s1] = top
    return out


def main(ref_dir: str) -> None:
    sys.path.insert(0, ref_dir)
    import kernel_sm121 as ks

    out = {}
    for name, (m, dt, scale, base, hc, iters, eps) in sinkhorn_cases().items():
        mt = (torch.from_numpy(m.view(np.int16)).view(torch.bfloat16) if dt == "bf16" else torch.from_numpy(m))
        pre, post, comb = ks.hc_split_sinkhorn(mt, torch.from_numpy(scale), torch.from_numpy(base), hc, iters, eps)
        out[f"hc/{name}/pre"] = pre.numpy()
        out[f"hc/{name}/post"] = post.numpy()
        out[f"hc/{name}/comb"] = comb.numpy()
    for name, (q, kv, sink, idx, scale, chunk) in sparse_attn_cases().items():
        ks.SPARSE_ATTN_CHUNK = chunk
        o = ks.sparse_attn(torch.from_numpy(q), torch.from_numpy(kv), torch.from_numpy(sink), torch.from_numpy(idx),
                           scale)
        out[f"sa/{name}/out"] = o.numpy()
    for name, (q, kv, w, topk, ratio, start_pos, offset) in indexer_cases().items():
        top = indexer_reference(torch.from_numpy(q), torch.from_numpy(kv), torch.from_numpy(w), topk, ratio,
                                start_pos, offset)
        out[f"ix/{name}/topk"] = top.numpy()
    path = os.path.join(HERE, "golden_attn.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("BS_REFERENCE_DIR", "")
    if not ref:
        sys.exit("usage: make_golden_attn.py <reference project directory> (or set BS_REFERENCE_DIR)")
    main(ref)
