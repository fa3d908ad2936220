"""Tensor-parallel (column-sharded) fp8_gemm / fp4_gemm with the all-gather
fused into the GEMM epilogue.

Rank r of g holds the weight rows [r*N/g, (r+1)*N/g) of B (and the matching
rows of its scales) and computes that column slice of C = A x B^T.  Instead
of writing the slice to a local buffer and all-gathering it with NCCL
(followed by a column interleave), every output tile is stored by the GEMM
epilogue straight into each rank's copy of C, mapped into this process
through symmetric memory; the NVLink transfer overlaps the remaining math.
A symmetric-memory barrier after the kernel makes every rank's slice
visible everywhere.  The barrier is the library's own
(bs_peer_barrier_counted: epoch flags in symmetric memory, the epoch counted
on the device so calls can be captured in CUDA graphs, bounded waits that
report a device-side timeout instead of trapping).

Two symmetric output buffers alternate between calls: every rank passes the
barrier of call i before any rank can start call i+1, so call i+1's stores
(into the other buffer) never touch the C of call i that a slower rank may
still be reading.  The C returned by a call is valid until the call after
next.

The weight sharding is the reference's TP split of the dense projections
(column-parallel linear layers; weight rows of one rank are contiguous),
with the all-gather that the reference would perform through NCCL.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

__all__ = ["TPGemm", "column_range", "shard_weight"]


def column_range(N: int, world: int, rank: int, align: int = 128):
    """Columns [c0, c1) of rank `rank`; N must split into 128-aligned slices
    (one fp8 weight-scale block row per 128 columns)."""
    if N % (world * align):
        raise ValueError(f"N={N} does not split into {world} slices of a multiple of {align} columns")
    n = N // world
    return rank * n, (rank + 1) * n


def shard_weight(b, b_s, world: int, rank: int, fp4: bool = False):
    """Rank `rank`'s rows of a full weight [N, ...] and of its scales (fp4:
    per-row ue8m0 [N, K/32]; fp8: per-128-row blocks [N/128, K/128])."""
    c0, c1 = column_range(b.shape[0], world, rank)
    if fp4:
        return b[c0:c1].contiguous(), b_s[c0:c1].contiguous()
    return b[c0:c1].contiguous(), b_s[c0 // 128:c1 // 128].contiguous()


class TPGemm:
    """C[M, N] (bf16, on every rank) = dequant(a) x dequant(b)^T with b
    column-sharded over ``group``.

    ``fp4`` selects the fp4_gemm form (b packed e2m1 [N/g, K/2], b_s ue8m0
    [N/g, K/32]); otherwise fp8_gemm (b e4m3 [N/g, K], b_s [N/g/128, K/128]).
    """

    def __init__(self, M: int, N: int, K: int, group=None, device=None, fp4: bool = False):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > 8:
            raise NotImplementedError("the fused all-gather writes to at most 8 ranks")
        self.M, self.N, self.K, self.fp4 = M, N, K, fp4
        self.col0, c1 = column_range(N, self.world, self.rank)
        self.n_local = c1 - self.col0
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.lib = _lib.load()
        name = self.group.group_name
        self.bufs, self.handles, self.ptrs = [], [], []
        order = [self.rank] + [q for q in range(self.world) if q != self.rank]
        for _ in range(2):
            t = symm_mem.empty(M, N, dtype=torch.bfloat16, device=self.device)
            h = symm_mem.rendezvous(t, name)
            arr = (ctypes.c_void_p * self.world)(*[self._peer_ptr(t, h, q) for q in order])
            self.bufs.append(t)
            self.handles.append(h)
            self.ptrs.append(arr)
        # barrier flags: rank q's array of `world` epochs, indexed by rank
        self.flags = symm_mem.empty(self.world, dtype=torch.int64, device=self.device)
        fh = symm_mem.rendezvous(self.flags, name)
        self.handles.append(fh)
        self.flag_ptrs = (ctypes.c_void_p * self.world)(*[self._peer_ptr(self.flags, fh, q)
                                                          for q in range(self.world)])
        self.epoch_ctr = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.flags.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.calls = 0
        self._fn = self.lib.bs_fp4_gemm_allgather if fp4 else self.lib.bs_fp8_gemm_allgather

    def _peer_ptr(self, t, h, q):
        # a tensor sits at the same offset inside every rank's symmetric
        # allocation; check that it lies inside this rank's buffer before
        # deriving a peer address from the offset
        base = h.buffer_ptrs[self.rank]
        off = t.data_ptr() - base
        nbytes = t.numel() * t.element_size()
        if off < 0 or off + nbytes > h.buffer_size:
            raise RuntimeError(f"symmetric tensor at offset {off} (+{nbytes} B) outside its {h.buffer_size}-byte buffer")
        return h.buffer_ptrs[q] + off

    def shard(self, b: torch.Tensor, b_s: torch.Tensor):
        """This rank's rows of the full weight and its scales."""
        return shard_weight(b, b_s, self.world, self.rank, self.fp4)

    def __call__(self, a: torch.Tensor, a_s: torch.Tensor, b_local: torch.Tensor, b_s_local: torch.Tensor,
                 stream=None) -> torch.Tensor:
        """a e4m3 [M, K], a_s [M, K/128] (fp32 or e8m0), this rank's weight
        shard -> the full C [M, N] on this rank (valid until the call after
        next)."""
        M, K = a.shape
        if M != self.M or K != self.K:
            raise ValueError(f"a is [{M}, {K}], expected [{self.M}, {self.K}]")
        if not (a.is_cuda and b_local.is_cuda):
            raise ValueError("tp gemm: CUDA tensors only (there is no CPU fallback)")
        i = self.calls & 1
        self.calls += 1
        st = stream if stream is not None else torch.cuda.current_stream(self.device)
        as_dt = _lib.DT_E8M0 if a_s.dtype == torch.uint8 or "float8_e8m0" in str(a_s.dtype) else _lib.DT_F32
        if self.fp4:
            bs_dt = _lib.DT_E8M0
        else:
            bs_dt = _lib.DT_E8M0 if b_s_local.dtype == torch.uint8 or "float8_e8m0" in str(b_s_local.dtype) \
                else _lib.DT_F32
        with torch.cuda.stream(st):
            _lib.check(self._fn(a.data_ptr(), a_s.data_ptr(), as_dt, b_local.data_ptr(), b_s_local.data_ptr(), bs_dt,
                                M, self.n_local, K, self.ptrs[i], self.world, self.N, self.col0, st.cuda_stream))
            # every rank's slice has landed in every rank's buffer i
            _lib.check(self.lib.bs_peer_barrier_counted(self.flag_ptrs, self.world, self.rank,
                                                        self.epoch_ctr.data_ptr(), st.cuda_stream))
        return self.bufs[i]

    def close(self):
        """Drop the symmetric buffers (before the process group is destroyed)."""
        self.bufs.clear()
        self.handles.clear()
        self.ptrs.clear()
        self.flags = None
