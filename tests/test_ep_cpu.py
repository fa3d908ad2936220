"""Expert-parallel MoE exchange logic on 2 and 4 gloo ranks (CPU, no GPU).

Each rank owns 1/world of the tokens and of the experts; rows travel by
all-to-all to the expert owners and back.  The skewed cases route every
token to the first top-k experts, so the other ranks receive no rows.  The kernels are numpy stand-ins
(tests/ep_cpu_ops.py), so this checks the counts exchange, the split sizes,
the (source, expert) -> expert-major regrouping, the arrival-order return and
the combine indexing against the single-process oracle layer.
"""

from __future__ import annotations

import importlib
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case(T, H, inter, E, topk, skew):
    import cases
    from oracle import blockscaled as ob
    m = cases.moe_case_small(T=T, H=H, inter=inter, E=E, topk=topk, seed=21)
    if skew:
        m["logits"] = m["logits"].copy()
        m["logits"][:, :topk] += 20.0
        m["idx"], m["w"] = ob.moe_route(m["logits"], topk)
    return m


def _worker(rank, world, port, q, T, H, inter, E, topk, skew):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    sys.path.insert(0, os.path.join(HERE, "golden"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ep_cpu_ops import CpuWeights, NumpyOps
        ep = importlib.import_module("deepseek-v4-experimental-platform-on-dgx-spark_b200.ep")
        m = _case(T, H, inter, E, topk, skew)
        e0, e1 = ep.expert_range(E, world, rank)
        W = CpuWeights(m["w13"][e0:e1], m["w13_s"][e0:e1], m["w2"][e0:e1], m["w2_s"][e0:e1])
        tl = T // world
        x = torch.from_numpy(m["x"][rank * tl:(rank + 1) * tl].view(np.int16)).view(torch.bfloat16)
        logits = torch.from_numpy(m["logits"][rank * tl:(rank + 1) * tl])
        layer = ep.EPMoE(W, E, topk, max_tokens=tl, ops=NumpyOps(), device=torch.device("cpu"))
        out = layer.forward(x, logits)
        q.put((rank, out.view(torch.int16).numpy().copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,skew", [(2, False), (4, False), (2, True), (4, True)])
def test_ep_ranks_match_single_process_oracle(world, skew):
    sys.path.insert(0, os.path.join(HERE, "golden"))
    from oracle import blockscaled as ob
    T, H, inter, E, topk = 16, 256, 128, 4, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, T, H, inter, E, topk, skew)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    out = np.concatenate([res[r] for r in range(world)]).view(np.uint16)
    m = _case(T, H, inter, E, topk, skew)
    ref = ob.moe_layer(m["x"], m["idx"], m["w"], m["w13"], m["w13_s"], m["w2"], m["w2_s"])
    o = ob.bf16_to_f32(out).astype(np.float64)
    r = ob.bf16_to_f32(ref).astype(np.float64)
    assert np.linalg.norm(o - r) / np.linalg.norm(r) < 1e-3
