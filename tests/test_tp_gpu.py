"""Tensor-parallel GEMM with the all-gather fused into the epilogue, on 2 GPUs.

Runs as two spawned ranks when at least two GPUs are visible; skipped
otherwise.  Each rank computes its column slice and stores it into both
ranks' symmetric output buffers; after the call, every rank's full C must be
bit-identical to the single-GPU GEMM of the whole weight (same kernel, same
per-tile arithmetic).  Two calls exercise both alternating output buffers.
"""

from __future__ import annotations

import importlib
import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
PKG = "deepseek-v4-experimental-platform-on-dgx-spark_b200"


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _problem(dev, M, N, K, fp4, seed):
    pkg = importlib.import_module(PKG)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
    a, a_s = pkg.act_quant(x, 128)
    if fp4:
        b = torch.randint(0, 256, (N, K // 2), generator=g, device=dev, dtype=torch.uint8)
        b_s = 127 - torch.randint(0, 7, (N, K // 32), generator=g, device=dev, dtype=torch.uint8)
    else:
        b = (torch.randn(N, K, generator=g, device=dev) * 4).clamp(-448, 448).to(torch.float8_e4m3fn)
        b_s = torch.rand(N // 128, K // 128, generator=g, device=dev) + 0.25
    return a, a_s, b, b_s


def _single(pkg, a, a_s, b, b_s, fp4):
    L = pkg._lib
    lib = L.load()
    M, K = a.shape
    N = b.shape[0]
    c = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    fn = lib.bs_fp4_gemm if fp4 else lib.bs_fp8_gemm
    L.check(fn(a.data_ptr(), a_s.data_ptr(), L.DT_F32, b.data_ptr(), b_s.data_ptr(),
               L.DT_E8M0 if fp4 else L.DT_F32, M, N, K, c.data_ptr(), torch.cuda.current_stream().cuda_stream))
    return c


def _worker(rank, world, port, q, M, N, K, fp4):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(HERE))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    layer = None
    try:
        pkg = importlib.import_module(PKG)
        tp = importlib.import_module(PKG + ".tp")
        a, a_s, b, b_s = _problem(dev, M, N, K, fp4, 11)
        ref = _single(pkg, a, a_s, b, b_s, fp4)
        layer = tp.TPGemm(M, N, K, device=dev, fp4=fp4)
        b_loc, s_loc = layer.shard(b, b_s)
        outs = []
        for i in range(3):
            c = layer(a, a_s, b_loc, s_loc)
            outs.append(c.clone())
        torch.cuda.synchronize()
        pkg._lib.device_error_check()
        same = [bool(torch.equal(o.view(torch.int16), ref.view(torch.int16))) for o in outs]
        q.put((rank, same))
        dist.barrier()
    finally:
        if layer is not None:
            layer.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("M,N,K,fp4", [(512, 1024, 1024, False), (300, 2048, 512, False), (256, 1024, 1024, True),
                                       (48, 512, 1024, False)])
def test_tp_allgather_two_gpus_match_single_gpu(M, N, K, fp4):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, M, N, K, fp4)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        assert all(res[r]), f"rank {r}: fused TP output differs from the single-GPU GEMM {res[r]}"
