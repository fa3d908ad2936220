"""Expert-parallel MoE layer across the GPUs of one node.

Experts are split into contiguous ranges, rank r owning experts
[r*E/g, (r+1)*E/g) -- the same ranges as the reference's loader
(weight_loader.py:112-139).  Tokens are split too: each rank routes and
quantises its own tokens, sends every (token, expert) row to the rank that
owns the expert, runs the grouped expert GEMMs on what it received, and gets
the expert outputs back for its weighted combine.  In the reference every
rank sees all tokens and the partial MoE outputs are all-reduced instead.

Two transports move the rows:

* ``peer`` (default on GPUs): over NVLink peer memory, with no NCCL call and
  no host round trip.  The receive buffers, the count matrix and the return
  buffer live in symmetric memory mapped by every rank.  Each rank pushes its
  per-expert counts to all ranks, plans from the full count matrix where its
  rows land at the owners, writes every row (with its scales and a return
  address) straight to its final expert-major place in the owner's buffer,
  and the owner's W2 epilogue stores each output row straight back into the
  source rank's return buffer.  Three bounded barrier kernels
  (bs_peer_barrier) order the steps.
* ``nccl`` (and the CPU tests on gloo):
  1. counts      all-to-all of the per-(destination, local expert) row counts
  2. dispatch    all-to-all-v of e4m3 rows (H bytes) and their ue8m0 scales
  3. return      all-to-all-v of the bf16 expert outputs, in arrival order
  The row counts are needed on the host for the variable-size exchanges, so
  a layer costs one small device-to-host copy.

Both transports put the rows of one expert in the same order (source rank,
then the source's expert-sorted order), so they give identical results.

The kernels (quantise, route, scan, dispatch, regroup, grouped GEMMs,
combine) are reached through ``ops``, an object with the methods of
:class:`CudaOps`; the CPU tests substitute a numpy implementation so that the
exchange logic runs on gloo ranks without a GPU.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib

__all__ = ["CudaOps", "EPMoE", "expert_range"]


def expert_range(E: int, world: int, rank: int):
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    n = E // world
    return rank * n, (rank + 1) * n


class CudaOps:
    """The MoE kernels of the CUDA library, on the current stream."""

    def __init__(self, device):
        self.device = device
        self.lib = _lib.load()

    def _st(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def quantise(self, x, xq, xs):
        T, H = x.shape
        _lib.check(self.lib.bs_act_quant(x.data_ptr(), _lib.DT_BF16, T, H, 128, 1, xq.data_ptr(), xs.data_ptr(),
                                         _lib.DT_E8M0, self._st()))

    def route(self, logits, topk, idx, w, counts):
        T, E = logits.shape
        _lib.check(self.lib.bs_moe_route(logits.data_ptr(), T, E, topk, idx.data_ptr(), w.data_ptr(),
                                         counts.data_ptr(), self._st()))

    def scan(self, counts, offsets, chunk_prefix, cursor):
        _lib.check(self.lib.bs_moe_scan(counts.data_ptr(), counts.numel(), offsets.data_ptr(),
                                        chunk_prefix.data_ptr(), cursor.data_ptr(), self._st()))

    def dispatch(self, idx, offsets, chunk_prefix, cursor, xq, xs, rows, rows_sc, pos_of):
        T, topk = idx.shape
        H = xq.shape[1]
        _lib.check(self.lib.bs_moe_dispatch(idx.data_ptr(), T, topk, offsets.data_ptr(), chunk_prefix.data_ptr(),
                                            cursor.data_ptr(), xq.data_ptr(), xs.data_ptr(), H, rows.data_ptr(),
                                            None, rows_sc.data_ptr(), pos_of.data_ptr(), self._st()))

    def regroup(self, recv_counts, n_src, E_loc, n_rows, rows_in, sc_in, rows_out, rows_sp, rowmap, offsets,
                chunk_prefix, scratch):
        H = rows_in.shape[1]
        _lib.check(self.lib.bs_moe_regroup(recv_counts.data_ptr(), n_src, E_loc, n_rows, rows_in.data_ptr(),
                                           sc_in.data_ptr(), H, rows_out.data_ptr(), rows_sp.data_ptr(),
                                           rowmap.data_ptr(), offsets.data_ptr(), chunk_prefix.data_ptr(),
                                           scratch.data_ptr(), self._st()))

    def experts(self, weights, n_rows, rows, rows_sp, offsets, chunk_prefix, rowmap, hq, hs_p, y):
        _lib.check(self.lib.bs_moe_experts(weights.E, n_rows, weights.H, weights.I, rows.data_ptr(),
                                           rows_sp.data_ptr(), offsets.data_ptr(), chunk_prefix.data_ptr(),
                                           weights.w13.data_ptr(), weights.w13_sp.data_ptr(),
                                           weights.w2.data_ptr(), weights.w2_sp.data_ptr(), rowmap.data_ptr(),
                                           hq.data_ptr(), hs_p.data_ptr(), y.data_ptr(), self._st()))

    def combine(self, y, pos_of, w, out):
        T, topk = pos_of.shape
        H = out.shape[1]
        _lib.check(self.lib.bs_moe_combine(y.data_ptr(), pos_of.data_ptr(), w.data_ptr(), T, topk, H,
                                           out.data_ptr(), self._st()))

    def chunk_capacity(self, rows, E):
        return int(self.lib.bs_moe_chunk_capacity(rows, E))

    # peer-memory transport (lists: one device pointer per rank, index = rank)
    def counts_push(self, counts, rank, n_ranks, cnt_ptrs):
        _lib.check(self.lib.bs_ep_counts_push(counts.data_ptr(), counts.numel(), rank, n_ranks, cnt_ptrs, self._st()))

    def plan(self, cnt_all, rank, send_pos0, loc_off, loc_chunks):
        n_ranks, E = cnt_all.shape
        _lib.check(self.lib.bs_ep_plan(cnt_all.data_ptr(), n_ranks, E, rank, send_pos0.data_ptr(), loc_off.data_ptr(),
                                       loc_chunks.data_ptr(), self._st()))

    def rows_push(self, rows, rows_sc, offsets, send_pos0, E, rank, n_ranks, max_rows, rows_ptrs, sc_ptrs, ret_ptrs):
        _lib.check(self.lib.bs_ep_rows_push(rows.data_ptr(), rows_sc.data_ptr(), offsets.data_ptr(),
                                            send_pos0.data_ptr(), E, rows.shape[1], rank, n_ranks, max_rows,
                                            rows_ptrs, sc_ptrs, ret_ptrs, self._st()))

    def pack_scales(self, recv_sc, loc_off, loc_chunks, E_loc, H, max_rows, rows_sp):
        _lib.check(self.lib.bs_ep_pack_scales(recv_sc.data_ptr(), loc_off.data_ptr(), loc_chunks.data_ptr(), E_loc, H,
                                              max_rows, rows_sp.data_ptr(), self._st()))

    def experts_return(self, weights, capacity, rows, rows_sp, offsets, chunk_prefix, ret, y_ptrs, n_ranks, hq, hs_p):
        _lib.check(self.lib.bs_ep_experts_return(weights.E, capacity, weights.H, weights.I, rows.data_ptr(),
                                                 rows_sp.data_ptr(), offsets.data_ptr(), chunk_prefix.data_ptr(),
                                                 weights.w13.data_ptr(), weights.w13_sp.data_ptr(),
                                                 weights.w2.data_ptr(), weights.w2_sp.data_ptr(), ret.data_ptr(),
                                                 y_ptrs, n_ranks, hq.data_ptr(), hs_p.data_ptr(), self._st()))

    def barrier(self, flag_ptrs, rank, n_ranks, counter):
        # epoch kept on the device (counter), so the layer can be captured in a CUDA graph
        _lib.check(self.lib.bs_peer_barrier_counted(flag_ptrs, n_ranks, rank, counter.data_ptr(), self._st()))


class EPMoE:
    """One MoE layer, expert-parallel over ``group``.

    ``weights`` holds this rank's experts only (any object with E, H, I and
    the packed weight / scale tensors, e.g. ``moe.MoEWeights``).  Buffers are
    sized for ``max_tokens`` tokens per rank; the receive side is sized for
    the worst case (every token of every rank routed to this rank).
    """

    def __init__(self, weights, E_total: int, topk: int, max_tokens: int, group=None, ops=None,
                 device=None, transport: str = "auto"):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = E_total
        self.E_loc = E_total // self.world
        if weights.E != self.E_loc:
            raise ValueError(f"rank {self.rank} holds {weights.E} experts, expected {self.E_loc}")
        self.w = weights
        self.topk = topk
        self.H, self.I = weights.H, weights.I
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.ops = ops if ops is not None else CudaOps(self.device)
        H, I, dev = self.H, self.I, self.device
        R = max_tokens * topk                   # rows this rank sends at most
        RR = R * self.world                     # rows this rank can receive at most
        u8, i32 = torch.uint8, torch.int32
        self.max_tokens = max_tokens
        self.xq = torch.empty(max_tokens, H, dtype=u8, device=dev)
        self.xs = torch.empty(max_tokens, H // 128, dtype=u8, device=dev)
        self.idx = torch.empty(max_tokens, topk, dtype=i32, device=dev)
        self.wts = torch.empty(max_tokens, topk, dtype=torch.float32, device=dev)
        self.pos_of = torch.empty(max_tokens, topk, dtype=i32, device=dev)
        self.counts = torch.empty(self.E, dtype=i32, device=dev)
        self.offsets = torch.empty(self.E + 1, dtype=i32, device=dev)
        self.chunks = torch.empty(self.E + 1, dtype=i32, device=dev)
        self.cursor = torch.empty(self.E, dtype=i32, device=dev)
        self.rows = torch.empty(R, H, dtype=u8, device=dev)
        self.rows_sc = torch.empty(R, H // 128, dtype=torch.int32, device=dev)
        nch = self.ops.chunk_capacity(RR, self.E_loc)
        self.grp_sp = torch.empty(nch * (H // 128) * 512, dtype=u8, device=dev)
        self.loc_off = torch.empty(self.E_loc + 1, dtype=i32, device=dev)
        self.loc_chunks = torch.empty(self.E_loc + 1, dtype=i32, device=dev)
        self.hq = torch.empty(RR, I, dtype=u8, device=dev)
        self.hs_p = torch.empty(nch * (I // 128) * 512, dtype=u8, device=dev)
        if transport == "auto":
            transport = "peer" if isinstance(self.ops, CudaOps) and self.world <= 8 else "nccl"
        if transport not in ("peer", "nccl"):
            raise ValueError(f"transport {transport!r}: expected 'peer', 'nccl' or 'auto'")
        self.transport = transport
        self.R, self.RR = R, RR
        if transport == "peer":
            self._init_peer(R, RR)
        else:
            self.recv_counts = torch.empty(self.world * self.E_loc, dtype=i32, device=dev)
            self.recv_rows = torch.empty(RR, H, dtype=u8, device=dev)
            self.recv_sc = torch.empty(RR, H // 128, dtype=torch.int32, device=dev)
            self.grp_rows = torch.empty(RR, H, dtype=u8, device=dev)
            self.rowmap = torch.empty(RR, dtype=i32, device=dev)
            self.scratch = torch.empty(2 * self.world * self.E_loc + 1, dtype=i32, device=dev)
            self.y_recv = torch.empty(RR, H, dtype=torch.bfloat16, device=dev)
            self.y_back = torch.empty(R, H, dtype=torch.bfloat16, device=dev)

    def _init_peer(self, R, RR):
        """Symmetric buffers that peers write, and their per-rank pointer lists."""
        import ctypes
        import torch.distributed._symmetric_memory as symm_mem
        H, dev, n, me = self.H, self.device, self.world, self.rank
        # peers write into these buffers at positions sized by their own
        # max_tokens: every rank must use the same value
        mt = torch.tensor([self.max_tokens, -self.max_tokens], dtype=torch.int64, device=dev)
        dist.all_reduce(mt, op=dist.ReduceOp.MAX, group=self.group)
        if int(mt[0]) != -int(mt[1]):
            raise ValueError("peer transport: max_tokens differs between ranks")
        name = (self.group if self.group is not None else dist.group.WORLD).group_name
        self._handles = []

        def sym(*shape, dtype):
            t = symm_mem.empty(*shape, dtype=dtype, device=dev)
            h = symm_mem.rendezvous(t, name)
            base = h.buffer_ptrs[me]
            off = t.data_ptr() - base
            if off < 0 or off + t.numel() * t.element_size() > h.buffer_size:
                raise RuntimeError("symmetric tensor outside its buffer")
            self._handles.append(h)
            return t, (ctypes.c_void_p * n)(*[h.buffer_ptrs[q] + off for q in range(n)])

        self.cnt_all, self.cnt_ptrs = sym(n, self.E, dtype=torch.int32)          # [src][e] counts
        self.recv_rows_p, self.rows_ptrs = sym(RR, H, dtype=torch.uint8)        # expert-major rows
        self.recv_sc_p, self.sc_ptrs = sym(RR, H // 128, dtype=torch.int32)     # their scale words
        self.recv_ret, self.ret_ptrs = sym(RR, dtype=torch.int32)                # src << 24 | src row
        self.y_back, self.y_ptrs = sym(R, H, dtype=torch.bfloat16)              # outputs returned here
        self.flags, self.flag_ptrs = sym(n, dtype=torch.int64)                    # barrier epochs
        self.send_pos0 = torch.empty(self.E, dtype=torch.int32, device=dev)
        self.epoch_ctr = torch.zeros(1, dtype=torch.int64, device=dev)
        self.flags.zero_()
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    def _barrier(self):
        self.ops.barrier(self.flag_ptrs, self.rank, self.world, self.epoch_ctr)

    def close(self):
        """Release the symmetric buffers (before the process group is destroyed)."""
        for a in ("cnt_all", "recv_rows_p", "recv_sc_p", "recv_ret", "y_back", "flags"):
            if hasattr(self, a):
                setattr(self, a, None)
        self._handles = []

    def forward(self, x: torch.Tensor, logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """x bf16 [T, H] (this rank's tokens), logits fp32 [T, E] -> bf16 [T, H]."""
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > max_tokens={self.max_tokens}")
        ops, g, El, k = self.ops, self.group, self.E_loc, self.topk
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.bfloat16, device=x.device)
        xq, xs = self.xq[:T], self.xs[:T]
        idx, wts, pos_of = self.idx[:T], self.wts[:T], self.pos_of[:T]
        ops.quantise(x.contiguous(), xq, xs)
        ops.route(logits.contiguous(), k, idx, wts, self.counts)
        ops.scan(self.counts, self.offsets, self.chunks, self.cursor)
        ops.dispatch(idx, self.offsets, self.chunks, self.cursor, xq, xs, self.rows, self.rows_sc, pos_of)
        if self.transport == "peer":
            return self._exchange_peer(pos_of, wts, out, T)
        # 1. counts: send_counts[d*El + e] = rows for destination d's local expert e
        dist.all_to_all_single(self.recv_counts, self.counts, group=g)
        both = torch.cat([self.counts.view(self.world, El).sum(1), self.recv_counts.view(self.world, El).sum(1)])
        both = both.cpu().tolist()              # the layer's one device-to-host copy
        send = both[:self.world]
        recv = both[self.world:]
        n_send, n_recv = sum(send), sum(recv)
        # 2. rows and scales to the expert owners (rows are expert-sorted, so
        #    each destination's rows are contiguous and in rank order)
        dist.all_to_all_single(self.recv_rows[:n_recv], self.rows[:n_send], recv, send, group=g)
        dist.all_to_all_single(self.recv_sc[:n_recv], self.rows_sc[:n_send], recv, send, group=g)
        # 3. expert-major order, grouped GEMMs, outputs written in arrival order
        ops.regroup(self.recv_counts, self.world, El, n_recv, self.recv_rows, self.recv_sc, self.grp_rows,
                    self.grp_sp, self.rowmap, self.loc_off, self.loc_chunks, self.scratch)
        if n_recv:
            ops.experts(self.w, n_recv, self.grp_rows, self.grp_sp, self.loc_off, self.loc_chunks, self.rowmap,
                        self.hq, self.hs_p, self.y_recv)
        # 4. outputs back to the token owners, then the weighted combine
        # (bf16 rows moved as bytes: same data, and every backend supports uint8)
        dist.all_to_all_single(self.y_back[:n_send].view(torch.uint8), self.y_recv[:n_recv].view(torch.uint8),
                               send, recv, group=g)
        ops.combine(self.y_back, pos_of, wts, out)
        return out

    def _exchange_peer(self, pos_of, wts, out, T):
        ops, n, me, El = self.ops, self.world, self.rank, self.E_loc
        ops.counts_push(self.counts, me, n, self.cnt_ptrs)
        self._barrier()                                   # every rank holds the full count matrix
        ops.plan(self.cnt_all, me, self.send_pos0, self.loc_off, self.loc_chunks)
        ops.rows_push(self.rows, self.rows_sc, self.offsets, self.send_pos0, self.E, me, n, T * self.topk,
                      self.rows_ptrs, self.sc_ptrs, self.ret_ptrs)
        self._barrier()                                   # every row is at its owner
        ops.pack_scales(self.recv_sc_p, self.loc_off, self.loc_chunks, El, self.H, self.RR, self.grp_sp)
        ops.experts_return(self.w, self.RR, self.recv_rows_p, self.grp_sp, self.loc_off, self.loc_chunks,
                           self.recv_ret, self.y_ptrs, n, self.hq, self.hs_p)
        self._barrier()                                   # every output row is back at its source
        ops.combine(self.y_back, pos_of, wts, out)
        return out
