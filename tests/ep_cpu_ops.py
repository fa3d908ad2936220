"""numpy stand-ins for the MoE kernels, for CPU (gloo) tests of the
expert-parallel exchange logic.  Same buffer contracts as CudaOps; the math
comes from the oracle."""

from __future__ import annotations

import numpy as np
import torch

from oracle import blockscaled as ob

KTOK = 112


def _np(t):
    return t.numpy()


class CpuWeights:
    def __init__(self, w13, w13_s, w2, w2_s):
        self.E, two_i, hh = w13.shape
        self.I, self.H = two_i // 2, hh * 2
        self.w13, self.w13_s, self.w2, self.w2_s = w13, w13_s, w2, w2_s


class NumpyOps:
    def quantise(self, x, xq, xs):
        q, s = ob.act_quant(_np(x.view(torch.int16)).view(np.uint16), ob.DT_BF16, 128, "ue8m0", ob.DT_E8M0)
        _np(xq)[:] = q
        _np(xs)[:] = s

    def route(self, logits, topk, idx, w, counts):
        i, ww = ob.moe_route(_np(logits), topk)
        _np(idx)[:] = i
        _np(w)[:] = ww
        _np(counts)[:] = np.bincount(i.ravel(), minlength=counts.numel())

    def scan(self, counts, offsets, chunk_prefix, cursor):
        c = _np(counts)
        _np(offsets)[:] = np.concatenate([[0], np.cumsum(c)])
        _np(chunk_prefix)[:] = np.concatenate([[0], np.cumsum((c + KTOK - 1) // KTOK)])
        _np(cursor)[:] = 0

    def dispatch(self, idx, offsets, chunk_prefix, cursor, xq, xs, rows, rows_sc, pos_of):
        I, off, cur = _np(idx), _np(offsets), _np(cursor)
        for t in range(I.shape[0]):
            for k in range(I.shape[1]):
                e = I[t, k]
                p = off[e] + cur[e]
                cur[e] += 1
                _np(pos_of)[t, k] = p
                _np(rows)[p] = _np(xq)[t]
                _np(rows_sc)[p] = (_np(xs)[t].astype(np.uint32) * 0x01010101).view(np.int32)

    def regroup(self, recv_counts, n_src, E, n_rows, rows_in, sc_in, rows_out, rows_sp, rowmap, offsets,
                chunk_prefix, scratch):
        cnt = _np(recv_counts).reshape(n_src, E)
        src_off = np.concatenate([[0], np.cumsum(cnt.ravel())])
        dst = 0
        for e in range(E):
            _np(offsets)[e] = dst
            for s in range(n_src):
                g = s * E + e
                for i in range(cnt[s, e]):
                    j = src_off[g] + i
                    _np(rows_out)[dst] = _np(rows_in)[j]
                    _np(rowmap)[dst] = j
                    self.sc_rows = getattr(self, "sc_rows", {})
                    self.sc_rows[dst] = (_np(sc_in)[j].view(np.uint32) & 0xFF).astype(np.uint8)
                    dst += 1
        _np(offsets)[E] = dst

    def experts(self, W, n_rows, rows, rows_sp, offsets, chunk_prefix, rowmap, hq, hs_p, y):
        off = _np(offsets)
        for e in range(W.E):
            r0, r1 = off[e], off[e + 1]
            if r1 == r0:
                continue
            a = _np(rows)[r0:r1]
            a_s = np.stack([self.sc_rows[r] for r in range(r0, r1)])
            gu = ob.bf16_to_f32(ob.fp4_gemm(a, a_s, W.w13[e], W.w13_s[e], ob.DT_E8M0, ob.DT_E8M0))
            z = (ob.silu_f32(gu[:, :W.I]) * gu[:, W.I:]).astype(np.float32)
            q, qs = ob.act_quant(z, ob.DT_F32, 128, "ue8m0", ob.DT_E8M0)
            yy = ob.fp4_gemm(q, qs, W.w2[e], W.w2_s[e], ob.DT_E8M0, ob.DT_E8M0)
            for i, r in enumerate(range(r0, r1)):
                _np(y.view(torch.int16))[_np(rowmap)[r]] = yy[i].view(np.int16)

    def combine(self, y, pos_of, w, out):
        P, W_ = _np(pos_of), _np(w)
        Y = ob.bf16_to_f32(_np(y.view(torch.int16)).view(np.uint16))
        acc = np.zeros((P.shape[0], Y.shape[1]), np.float32)
        for t in range(P.shape[0]):
            for k in range(P.shape[1]):
                acc[t] += W_[t, k] * Y[P[t, k]]
        _np(out.view(torch.int16))[:] = ob.f32_to_bf16(acc).view(np.int16)

    def chunk_capacity(self, rows, E):
        return rows // KTOK + E
