"""ctypes binding of the C ABI in include/bsgemm.h (libbsgemm.so, built in-tree).

There is no fallback: if the shared library is missing or cannot be loaded,
every call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbsgemm.so")

# dtype tags (bs_dtype)
DT_F32, DT_BF16, DT_F16, DT_E4M3, DT_E8M0, DT_E2M1X2 = 0, 1, 2, 3, 4, 5
# status codes
BS_OK, BS_ERR_INVALID_ARG, BS_ERR_UNSUPPORTED, BS_ERR_CUDA, BS_ERR_DEVICE_TIMEOUT = 0, 1, 2, 3, 4

_c_void_p, _i64, _i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int

# name -> argtypes, exactly the declarations of include/bsgemm.h
SIGNATURES = {
    "bs_version": [],
    "bs_last_error": [],
    "bs_device_error_check": [],
    "bs_act_quant": [_c_void_p, _i32, _i64, _i64, _i32, _i32, _c_void_p, _c_void_p, _i32, _c_void_p],
    "bs_act_quant_inplace": [_c_void_p, _i32, _i64, _i64, _i32, _i32, _c_void_p],
    "bs_fp4_act_quant_inplace": [_c_void_p, _i32, _i64, _i64, _i32, _c_void_p],
    "bs_fp8_gemm": [_c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p, _i32, _i64, _i64, _i64, _c_void_p, _c_void_p],
    "bs_fp4_gemm": [_c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p, _i32, _i64, _i64, _i64, _c_void_p, _c_void_p],
    "bs_fp4_weights_to_bf16": [_c_void_p, _c_void_p, _i64, _i64, _c_void_p, _c_void_p],
    "bs_e4m3_rows_to_bf16": [_c_void_p, _c_void_p, _i32, _i64, _i64, _c_void_p, _c_void_p],
    "bs_sparse_attn_workspace_size": [_i64, _i64, _i32, _i32, _i32],
    "bs_sparse_attn": [_c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p, _i32, _i64, _i64, _i32, _i32, _i64, _i32,
                       ctypes.c_float, _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p],
    "bs_indexer_topk_workspace_size": [_i64, _i64],
    "bs_indexer_topk": [_c_void_p, _c_void_p, _i32, _c_void_p, _i64, _i32, _i32, _i64, _i32, _i32, _i64, _i64,
                        _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p],
    "bs_e4m3_blocks_to_bf16": [_c_void_p, _c_void_p, _i32, _i64, _i64, _c_void_p, _c_void_p],
    "bs_hc_split_sinkhorn": [_c_void_p, _i32, _c_void_p, _c_void_p, _i64, _i32, _i32, ctypes.c_float, _c_void_p,
                             _c_void_p, _c_void_p, _c_void_p],
    "bs_fp8_gemm_allgather": [_c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p, _i32, _i64, _i64, _i64,
                              ctypes.POINTER(_c_void_p), _i32, _i64, _i64, _c_void_p],
    "bs_fp4_gemm_allgather": [_c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p, _i32, _i64, _i64, _i64,
                              ctypes.POINTER(_c_void_p), _i32, _i64, _i64, _c_void_p],
    "bs_peer_barrier": [ctypes.POINTER(_c_void_p), _i32, _i32, _i64, _c_void_p],
    "bs_peer_barrier_counted": [ctypes.POINTER(_c_void_p), _i32, _i32, _c_void_p, _c_void_p],
    "bs_moe_pack_scales": [_c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p],
    "bs_moe_chunk_capacity": [_i64, _i32],
    "bs_moe_workspace_size": [_i64, _i32, _i32, _i32, _i32],
    "bs_moe_forward": [_c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p,
                       _c_void_p, _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p],
    "bs_moe_staged_workspace_size": [_i64, _i32, _i32, _i32, _i32],
    "bs_moe_forward_staged": [_c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p,
                              _c_void_p, _c_void_p, _c_void_p, ctypes.c_size_t, _c_void_p],
    "bs_moe_time_layer": [_c_void_p, _c_void_p],
    "bs_ep_moe_sizes": [_i64, _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(_i64)],
    "bs_ep_moe_forward": [_c_void_p, _c_void_p, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p,
                          _c_void_p, _c_void_p, _c_void_p, ctypes.POINTER(_c_void_p), _c_void_p, ctypes.c_size_t,
                          _c_void_p],
    "bs_moe_forward_noalloc": [_c_void_p, _c_void_p, _i64, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p,
                               _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    "bs_moe_gate": [_c_void_p, _c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p],
    "bs_moe_route": [_c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    "bs_moe_scan": [_c_void_p, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    "bs_moe_dispatch": [_c_void_p, _i64, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32,
                        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    "bs_moe_regroup": [_c_void_p, _i32, _i32, _i64, _c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p, _c_void_p,
                       _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    "bs_moe_experts": [_i32, _i64, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                       _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    "bs_moe_combine": [_c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p],
}
RESTYPES = {"bs_last_error": ctypes.c_char_p, "bs_moe_workspace_size": ctypes.c_size_t,
            "bs_moe_staged_workspace_size": ctypes.c_size_t, "bs_moe_chunk_capacity": ctypes.c_int64,
            "bs_moe_time_layer": None, "bs_sparse_attn_workspace_size": ctypes.c_size_t,
            "bs_indexer_topk_workspace_size": ctypes.c_size_t}


class BsError(RuntimeError):
    """A non-zero status from the library; ``code`` is the BS_ERR_* value."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[bsgemm status {code}] {msg}")
        self.code = code


_lock = threading.Lock()
_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(
                    f"{path} is missing: build it with `python {os.path.join(HERE, 'build.py')}` "
                    "(the block-scaled kernels have no CPU fallback)")
            lib = ctypes.CDLL(path)
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = RESTYPES.get(name, ctypes.c_int)
            _lib = lib
    return _lib


def check(status: int) -> None:
    if status != BS_OK:
        msg = load().bs_last_error().decode(errors="replace")
        if status == BS_ERR_INVALID_ARG:
            raise ValueError(f"[bsgemm] {msg}")
        if status == BS_ERR_UNSUPPORTED:
            raise NotImplementedError(f"[bsgemm] {msg}")
        raise BsError(status, msg)


def device_error_check() -> None:
    """Synchronise and raise if a kernel recorded a device-side error."""
    check(load().bs_device_error_check())
