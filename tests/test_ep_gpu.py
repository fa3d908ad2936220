"""Expert-parallel MoE on 2 GPUs (NCCL) vs the single-GPU layer on the same batch.

Runs as two spawned ranks when at least two GPUs are visible; skipped
otherwise.  Every rank routes its half of the tokens, exchanges rows with the
expert owners, and the gathered result must equal what one GPU computes with
all experts (same kernels, same per-row arithmetic).
"""

from __future__ import annotations

import importlib
import os
import socket
import sys

import numpy as np
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


def _problem(dev, T, H, I, E, seed, skew=False, topk=8):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g, device=dev)
    if skew:
        # every token's top-k are the first topk experts: ranks owning none of them receive nothing
        logits[:, :topk] += 20.0
    w13 = torch.randint(0, 256, (E, 2 * I, H // 2), generator=g, device=dev, dtype=torch.uint8)
    w13_s = 127 - torch.randint(0, 7, (E, 2 * I, H // 32), generator=g, device=dev, dtype=torch.uint8)
    w2 = torch.randint(0, 256, (E, H, I // 2), generator=g, device=dev, dtype=torch.uint8)
    w2_s = 127 - torch.randint(0, 7, (E, H, I // 32), generator=g, device=dev, dtype=torch.uint8)
    return x, logits, w13, w13_s, w2, w2_s


def _worker(rank, world, port, q, T, H, I, E, topk, transport, skew):
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
        ep = importlib.import_module(PKG + ".ep")
        moe = importlib.import_module(PKG + ".moe")
        x, logits, w13, w13_s, w2, w2_s = _problem(dev, T, H, I, E, 5, skew, topk)
        e0, e1 = ep.expert_range(E, world, rank)
        W = moe.MoEWeights(w13[e0:e1], w13_s[e0:e1], w2[e0:e1], w2_s[e0:e1])
        tl = T // world
        layer = ep.EPMoE(W, E, topk, max_tokens=tl, transport=transport)
        outs = []
        for _ in range(2):
            outs.append(layer.forward(x[rank * tl:(rank + 1) * tl], logits[rank * tl:(rank + 1) * tl]).clone())
        torch.cuda.synchronize()
        res = {"ep": [o.cpu().view(torch.int16).numpy() for o in outs]}
        if rank == 0:
            full = moe.moe_forward(x, logits, moe.MoEWeights(w13, w13_s, w2, w2_s), topk)
            res["ref"] = full.cpu().view(torch.int16).numpy()
        importlib.import_module(PKG + "._lib").device_error_check()
        q.put((rank, res))
        dist.barrier()
    except BaseException as exc:   # report at once instead of leaving the parent waiting
        q.put((rank, {"error": repr(exc)}))
        raise
    finally:
        if layer is not None and hasattr(layer, "close"):
            layer.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("transport", ["peer", "nccl"])
@pytest.mark.parametrize("T,H,I,E,topk,skew", [(64, 512, 256, 16, 4, False), (256, 4096, 2048, 32, 8, False),
                                               (64, 512, 256, 16, 4, True)])
def test_ep_matches_single_gpu(T, H, I, E, topk, skew, transport, world):
    """Expert-parallel layer on `world` GPUs (skipped when fewer are visible)
    gives the single-GPU layer's bits on the same batch, on two calls in a
    row; the skewed case routes every token to the first top-k experts, so
    the ranks owning none of them receive nothing."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, T, H, I, E, topk, transport, skew))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, v = q.get(timeout=240)
        assert "error" not in v, (r, v.get("error"))
        res[r] = v
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ref = res[0]["ref"].view(np.uint16)
    for call in range(2):
        ep = np.concatenate([res[r]["ep"][call] for r in range(world)]).view(np.uint16)
        r = (ref.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        o = (ep.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        err = np.linalg.norm(o - r) / np.linalg.norm(r)
        same = np.array_equal(ep, ref)
        print(f"EP{world} ({transport}) T={T} H={H} E={E} call {call}: rel_fro={err:.3e}, identical={same}")
        assert same
