"""bs_moe_forward_noalloc: the MoE layer for callers that cannot allocate.

Callers such as a host framework that owns all device memory, or a plugin
that must not call cudaMalloc, cannot hand the layer a workspace.  The
no-alloc entry point runs the same layer on a fixed scratch array inside the
library.  These tests call it through the C ABI and compare it bit for bit
with bs_moe_forward given a fresh workspace on the same inputs (both run the
same deterministic kernels).  The scratch keeps the previous call's
contents, so each case calls the entry point twice in a row, and a large
call is followed by smaller ones with other seeds, token counts and expert
counts: anything stale that leaked through the shared scratch would show
up as a difference.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from conftest import PKG_NAME

pytestmark = pytest.mark.gpu

def _lib():
    return importlib.import_module(PKG_NAME + "._lib")


def _make(T, H, inter, E, seed):
    mm = importlib.import_module(PKG_NAME + ".moe")
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g, device=dev)
    w13 = torch.randint(0, 256, (E, 2 * inter, H // 2), generator=g, device=dev, dtype=torch.uint8)
    w13_s = 127 - torch.randint(0, 7, (E, 2 * inter, H // 32), generator=g, device=dev, dtype=torch.uint8)
    w2 = torch.randint(0, 256, (E, H, inter // 2), generator=g, device=dev, dtype=torch.uint8)
    w2_s = 127 - torch.randint(0, 7, (E, H, inter // 32), generator=g, device=dev, dtype=torch.uint8)
    return x, logits, mm.MoEWeights(w13, w13_s, w2, w2_s)


def _with_workspace(x, logits, W, topk):
    L = _lib()
    lib = L.load()
    T, H = x.shape
    ws = torch.empty(lib.bs_moe_workspace_size(T, H, W.I, W.E, topk), dtype=torch.uint8, device=x.device)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    L.check(lib.bs_moe_forward(x.data_ptr(), logits.data_ptr(), T, H, W.I, W.E, topk, W.w13.data_ptr(),
                               W.w13_sp.data_ptr(), W.w2.data_ptr(), W.w2_sp.data_ptr(), out.data_ptr(),
                               ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream))
    return out


def _no_alloc(x, logits, W, topk, out):
    L = _lib()
    T, H = x.shape
    return L.load().bs_moe_forward_noalloc(x.data_ptr(), logits.data_ptr(), T, H, W.I, W.E, topk,
                                           W.w13.data_ptr(), W.w13_sp.data_ptr(), W.w2.data_ptr(),
                                           W.w2_sp.data_ptr(), out.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)


# largest first, then smaller calls with other seeds, sizes and expert counts
CASES = [(448, 4096, 2048, 64, 8, 1), (256, 4096, 2048, 32, 8, 2), (64, 512, 256, 16, 4, 3), (100, 384, 256, 4, 2, 4)]


def test_no_alloc_matches_workspace_entry_point():
    for T, H, inter, E, topk, seed in CASES:
        x, logits, W = _make(T, H, inter, E, seed=seed)
        ref = _with_workspace(x, logits, W, topk)
        for call in range(2):
            out = torch.full((T, H), float("nan"), dtype=torch.bfloat16, device="cuda")
            _lib().check(_no_alloc(x, logits, W, topk, out))
            torch.cuda.synchronize()
            same = torch.equal(out, ref)
            print(f"no-alloc T={T} H={H} I={inter} E={E} k={topk} call {call}: bit-equal={same}")
            assert torch.isfinite(out.float()).all()
            assert same, (T, H, inter, E, topk, call)
    _lib().device_error_check()


def test_no_alloc_rejects_sizes_beyond_its_scratch():
    L = _lib()
    lib = L.load()
    # 2048 tokens x top-8 at hidden 4096 needs far more than the 64 MiB scratch
    need = lib.bs_moe_workspace_size(2048, 4096, 2048, 256, 8)
    assert need > 64 * 2**20
    st = lib.bs_moe_forward_noalloc(None, None, 2048, 4096, 2048, 256, 8, None, None, None, None, None, None)
    assert st == L.BS_ERR_UNSUPPORTED
    assert b"scratch" in lib.bs_last_error()
