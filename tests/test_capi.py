"""The C-ABI library loads, exports every symbol include/bsgemm.h declares, and
rejects bad arguments with a status code and message (no GPU needed: argument
validation runs before any CUDA call)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT, import_pkg

HEADER = os.path.join(ROOT, "include", "bsgemm.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|size_t|void|const char\*)\s+(bs_\w+)\s*\(", src, re.M)))


@pytest.fixture(scope="module")
def lib():
    pkg = import_pkg()
    from importlib import import_module
    build = import_module(pkg.__name__ + ".build")
    build.build()
    return pkg._lib.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ["bs_version", "bs_last_error", "bs_device_error_check", "bs_act_quant", "bs_act_quant_inplace",
              "bs_fp4_act_quant_inplace", "bs_fp8_gemm", "bs_fp4_gemm", "bs_moe_workspace_size",
              "bs_moe_forward", "bs_moe_route", "bs_moe_scan", "bs_moe_dispatch", "bs_moe_regroup",
              "bs_moe_experts", "bs_moe_combine"]:
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    for s in declared_symbols():
        assert hasattr(lib, s), s
    pkg = import_pkg()
    assert set(pkg._lib.SIGNATURES) == set(declared_symbols())
    assert lib.bs_version() >= 100


def test_invalid_args_return_status(lib):
    pkg = import_pkg()
    L = pkg._lib
    # bad x dtype
    assert lib.bs_act_quant(None, 99, 4, 128, 128, 0, None, None, L.DT_F32, None) == L.BS_ERR_INVALID_ARG
    assert b"dtype" in lib.bs_last_error()
    # K not a multiple of block_size
    assert lib.bs_act_quant(None, L.DT_BF16, 4, 100, 128, 0, None, None, L.DT_F32, None) == L.BS_ERR_INVALID_ARG
    # non-power-of-two block size
    assert lib.bs_fp4_act_quant_inplace(None, L.DT_BF16, 4, 96, 48, None) == L.BS_ERR_UNSUPPORTED
    # GEMM: K not a multiple of 128
    assert lib.bs_fp4_gemm(None, None, L.DT_F32, None, None, L.DT_E8M0, 16, 256, 100, None, None) == L.BS_ERR_UNSUPPORTED
    # GEMM: fp4 weight scales must be e8m0
    assert lib.bs_fp4_gemm(None, None, L.DT_F32, None, None, L.DT_F32, 16, 256, 128, None, None) == L.BS_ERR_UNSUPPORTED
    # GEMM: null pointers
    assert lib.bs_fp8_gemm(None, None, L.DT_F32, None, None, L.DT_F32, 16, 256, 128, None, None) == L.BS_ERR_INVALID_ARG
    # empty problems are a no-op
    assert lib.bs_fp8_gemm(None, None, L.DT_F32, None, None, L.DT_F32, 0, 256, 128, None, None) == L.BS_OK
    assert lib.bs_act_quant(None, L.DT_BF16, 0, 128, 128, 0, None, None, L.DT_F32, None) == L.BS_OK
    # MoE: sizes
    assert lib.bs_moe_workspace_size(1024, 4096, 2048, 256, 8) > 100 * 2**20
    assert lib.bs_moe_workspace_size(16, 100, 2048, 256, 8) == 0
    assert lib.bs_moe_forward(None, None, 16, 4096, 2048, 2000, 8, None, None, None, None, None, None, 0,
                              None) == L.BS_ERR_UNSUPPORTED
    assert lib.bs_moe_forward(None, None, 16, 4096, 2048, 256, 8, None, None, None, None, None, None, 0,
                              None) == L.BS_ERR_INVALID_ARG


def test_python_check_maps_status(lib):
    pkg = import_pkg()
    L = pkg._lib
    with pytest.raises(ValueError):
        L.check(lib.bs_act_quant(None, 99, 4, 128, 128, 0, None, None, L.DT_F32, None))
    with pytest.raises(NotImplementedError):
        L.check(lib.bs_fp4_gemm(None, None, L.DT_F32, None, None, L.DT_F32, 16, 256, 128, None, None))


def test_cpu_tensors_rejected():
    import torch
    pkg = import_pkg()
    x = torch.zeros(4, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        pkg.act_quant(x)
    with pytest.raises(AssertionError):
        pkg.act_quant(torch.zeros(4, 100, dtype=torch.bfloat16))
    with pytest.raises(NotImplementedError):
        pkg.fp4_act_quant(torch.zeros(4, 32, dtype=torch.bfloat16), 32, False)


def test_multi_gpu_entry_points_validate_arguments(lib):
    """Tensor-parallel, barrier and expert-parallel entry points reject bad
    arguments before any CUDA call."""
    pkg = import_pkg()
    L = pkg._lib
    vp = ctypes.c_void_p
    nine = (vp * 9)(*([None] * 9))
    two = (vp * 2)(None, None)
    # fused all-gather GEMM: 1..8 output buffers, columns must fit the rows
    assert lib.bs_fp8_gemm_allgather(None, None, L.DT_F32, None, None, L.DT_F32, 16, 256, 128, nine, 9, 512, 0,
                                     None) == L.BS_ERR_UNSUPPORTED
    assert lib.bs_fp8_gemm_allgather(None, None, L.DT_F32, None, None, L.DT_F32, 16, 256, 128, None, 2, 512, 0,
                                     None) == L.BS_ERR_INVALID_ARG
    assert lib.bs_fp8_gemm_allgather(None, None, L.DT_F32, None, None, L.DT_F32, 16, 256, 128, two, 2, 512, 384,
                                     None) == L.BS_ERR_INVALID_ARG
    assert b"do not fit" in lib.bs_last_error()
    assert lib.bs_fp4_gemm_allgather(None, None, L.DT_F32, None, None, L.DT_E8M0, 0, 256, 128, two, 2, 512, 256,
                                     None) == L.BS_OK
    # barriers: rank range, positive epoch, a counter
    assert lib.bs_peer_barrier(two, 0, 0, 1, None) == L.BS_ERR_INVALID_ARG
    assert lib.bs_peer_barrier(two, 2, 2, 1, None) == L.BS_ERR_INVALID_ARG
    assert lib.bs_peer_barrier(two, 2, 0, 0, None) == L.BS_ERR_INVALID_ARG
    assert lib.bs_peer_barrier(two, 2, 0, 1, None) == L.BS_ERR_INVALID_ARG   # null flag arrays
    assert lib.bs_peer_barrier_counted(two, 2, 0, None, None) == L.BS_ERR_INVALID_ARG
    # expert-parallel layer: experts split evenly over 1..8 ranks, H a multiple of 256
    sizes = (ctypes.c_int64 * 7)()
    assert lib.bs_ep_moe_sizes(16, 4096, 2048, 255, 8, 2, sizes) == L.BS_ERR_UNSUPPORTED
    assert b"do not split" in lib.bs_last_error()
    assert lib.bs_ep_moe_sizes(16, 384, 256, 16, 4, 2, sizes) == L.BS_ERR_UNSUPPORTED
    assert lib.bs_ep_moe_sizes(16, 4096, 2048, 256, 8, 9, sizes) == L.BS_ERR_INVALID_ARG
    assert lib.bs_ep_moe_sizes(16, 4096, 2048, 256, 8, 2, None) == L.BS_ERR_INVALID_ARG
    assert lib.bs_ep_moe_sizes(16, 4096, 2048, 256, 8, 2, sizes) == L.BS_OK
    assert sizes[1] == 8 * 2 * 256                    # count matrix: [ranks][E] 64-bit words
    assert sizes[2] == 2 * 16 * 8 * 4096              # receive rows: ranks x max_tokens x topk rows of H bytes
    assert sizes[5] == 16 * 8 * 4096 * 2              # returned bf16 rows of this rank's tokens
    assert sizes[0] > 0 and sizes[6] > 0
    peers = (ctypes.c_void_p * 12)()
    assert lib.bs_ep_moe_forward(None, None, 17, 16, 4096, 2048, 256, 8, 0, 2, None, None, None, None, None, peers,
                                 None, 0, None) == L.BS_ERR_INVALID_ARG      # more tokens than max_tokens
    assert lib.bs_ep_moe_forward(None, None, 0, 16, 4096, 2048, 256, 8, 2, 2, None, None, None, None, None, peers,
                                 None, 0, None) == L.BS_ERR_INVALID_ARG      # rank out of range
