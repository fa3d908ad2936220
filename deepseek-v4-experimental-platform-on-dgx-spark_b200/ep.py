"""Expert-parallel MoE layer across the GPUs of one node.

Experts are split into contiguous ranges, rank r owning experts
[r*E/g, (r+1)*E/g) -- the same ranges as the reference's loader
(weight_loader.py:112-139).  Tokens are split too: each rank routes and
quantises its own tokens, sends every (token, expert) row to the rank that
owns the expert, runs the grouped expert GEMMs on what it received, and gets
the expert outputs back for its weighted combine.  In the reference every
rank sees all tokens and the partial MoE outputs are all-reduced instead.

Two transports move the rows:

* ``peer`` (default on GPUs): the whole layer is one cooperative kernel of
  this library (bs_ep_moe_forward), with no NCCL call, no host round trip
  and no separate barrier: its front phase quantises and routes this rank's
  tokens, exchanges the per-expert counts through peer memory, and writes
  every (token, slot) row with its scales and a return address straight to
  its final expert-major place in the owning rank's receive buffer; its
  experts phase (W1|W3 and W2 grouped GEMMs, persistent) starts once every
  rank's rows are in and stores each output row straight back into the
  source rank's return buffer; its combine phase waits for every rank's
  returns.  The receive buffers, count matrix, return buffer
  and sync words live in symmetric memory mapped by every rank.
* ``nccl`` (and the CPU tests on gloo):
  1. counts      all-to-all of the per-(destination, local expert) row counts
  2. dispatch    all-to-all-v of e4m3 rows (H bytes) and their ue8m0 scales
  3. return      all-to-all-v of the bf16 expert outputs, in arrival order
  The row counts are needed on the host for the variable-size exchanges, so
  a layer costs one small device-to-host copy.

No row's result depends on where it sits among its expert's rows, so both
transports give the single-GPU layer's bits.

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


class EPMoE:
    """One MoE layer, expert-parallel over ``group``.

    ``weights`` holds this rank's experts only (any object with E, H, I and
    the packed weight / scale tensors, e.g. ``moe.MoEWeights``).  Buffers are
    sized for ``max_tokens`` tokens per rank (the same on every rank); the
    receive side is sized for the worst case (every token of every rank
    routed to this rank).
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
        self.max_tokens = max_tokens
        if transport == "auto":
            transport = "peer" if isinstance(self.ops, CudaOps) and self.world <= 8 else "nccl"
        if transport not in ("peer", "nccl"):
            raise ValueError(f"transport {transport!r}: expected 'peer', 'nccl' or 'auto'")
        self.transport = transport
        self.R = max_tokens * topk              # rows this rank sends at most
        self.RR = self.R * self.world           # rows this rank can receive at most
        if transport == "peer":
            self._init_peer()
        else:
            self._init_nccl()

    def _init_nccl(self):
        H, I, dev, topk, R, RR = self.H, self.I, self.device, self.topk, self.R, self.RR
        u8, i32 = torch.uint8, torch.int32
        mt = self.max_tokens
        self.xq = torch.empty(mt, H, dtype=u8, device=dev)
        self.xs = torch.empty(mt, H // 128, dtype=u8, device=dev)
        self.idx = torch.empty(mt, topk, dtype=i32, device=dev)
        self.wts = torch.empty(mt, topk, dtype=torch.float32, device=dev)
        self.pos_of = torch.empty(mt, topk, dtype=i32, device=dev)
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
        self.recv_counts = torch.empty(self.world * self.E_loc, dtype=i32, device=dev)
        self.recv_rows = torch.empty(RR, H, dtype=u8, device=dev)
        self.recv_sc = torch.empty(RR, H // 128, dtype=torch.int32, device=dev)
        self.grp_rows = torch.empty(RR, H, dtype=u8, device=dev)
        self.rowmap = torch.empty(RR, dtype=i32, device=dev)
        self.scratch = torch.empty(2 * self.world * self.E_loc + 1, dtype=i32, device=dev)
        self.y_recv = torch.empty(RR, H, dtype=torch.bfloat16, device=dev)
        self.y_back = torch.empty(R, H, dtype=torch.bfloat16, device=dev)

    def _init_peer(self):
        """The single-kernel layer (bs_ep_moe_forward): a local workspace and
        six symmetric buffers per rank that peers write (count matrix, receive
        rows, their packed scales, return addresses, returned outputs, sync
        words), with one pointer list over all ranks."""
        import ctypes
        import torch.distributed._symmetric_memory as symm_mem
        dev, n, me = self.device, self.world, self.rank
        lib = _lib.load()
        # peers write into these buffers at positions sized by their own
        # max_tokens, and count on the same CTAs per rank: every rank must
        # use the same max_tokens and have the same SM count
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        chk = torch.tensor([self.max_tokens, -self.max_tokens, sms, -sms], dtype=torch.int64, device=dev)
        dist.all_reduce(chk, op=dist.ReduceOp.MAX, group=self.group)
        if int(chk[0]) != -int(chk[1]) or int(chk[2]) != -int(chk[3]):
            raise ValueError("peer transport: max_tokens or the SM count differs between ranks")
        sizes = (ctypes.c_int64 * 7)()
        _lib.check(lib.bs_ep_moe_sizes(self.max_tokens, self.H, self.I, self.E, self.topk, n, sizes))
        self.ws = torch.zeros(sizes[0], dtype=torch.uint8, device=dev)
        name = (self.group if self.group is not None else dist.group.WORLD).group_name
        self._handles, self._sym = [], []
        ptrs = []
        for k in range(1, 7):
            t = symm_mem.empty(int(sizes[k]), dtype=torch.uint8, device=dev)
            t.zero_()
            h = symm_mem.rendezvous(t, name)
            off = t.data_ptr() - h.buffer_ptrs[me]
            if off < 0 or off + t.numel() > h.buffer_size:
                raise RuntimeError("symmetric tensor outside its buffer")
            self._handles.append(h)
            self._sym.append(t)
            ptrs += [h.buffer_ptrs[q] + off for q in range(n)]
        self.peer_ptrs = (ctypes.c_void_p * (6 * n))(*ptrs)
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    def close(self):
        """Release the symmetric buffers (before the process group is destroyed)."""
        self._sym = []
        self._handles = []

    def forward(self, x: torch.Tensor, logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """x bf16 [T, H] (this rank's tokens), logits fp32 [T, E] -> bf16 [T, H]."""
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > max_tokens={self.max_tokens}")
        ops, g, El, k = self.ops, self.group, self.E_loc, self.topk
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.bfloat16, device=x.device)
        if self.transport == "peer":
            return self._forward_peer(x.contiguous(), logits.contiguous(), out, T)
        xq, xs = self.xq[:T], self.xs[:T]
        idx, wts, pos_of = self.idx[:T], self.wts[:T], self.pos_of[:T]
        ops.quantise(x.contiguous(), xq, xs)
        ops.route(logits.contiguous(), k, idx, wts, self.counts)
        ops.scan(self.counts, self.offsets, self.chunks, self.cursor)
        ops.dispatch(idx, self.offsets, self.chunks, self.cursor, xq, xs, self.rows, self.rows_sc, pos_of)
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

    def _forward_peer(self, x, logits, out, T):
        w, lib = self.w, _lib.load()
        _lib.check(lib.bs_ep_moe_forward(
            x.data_ptr(), logits.data_ptr(), T, self.max_tokens, self.H, self.I, self.E, self.topk, self.rank,
            self.world, w.w13.data_ptr(), w.w13_sp.data_ptr(), w.w2.data_ptr(), w.w2_sp.data_ptr(), out.data_ptr(),
            self.peer_ptrs, self.ws.data_ptr(), self.ws.numel(),
            torch.cuda.current_stream(self.device).cuda_stream))
        return out
