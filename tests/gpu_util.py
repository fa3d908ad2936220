"""numpy <-> CUDA tensor helpers for the GPU parity tests (bit-preserving)."""

from __future__ import annotations

import numpy as np
import torch


def cuda_bf16(u16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16).cuda()


def cuda_u8(u8: np.ndarray, dtype=torch.uint8) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(u8)).cuda().view(dtype)


def cuda_f32(f: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(f, dtype=np.float32)).cuda()


def cuda_x(x: np.ndarray, xdt: str) -> torch.Tensor:
    return cuda_bf16(x) if xdt == "bf16" else cuda_f32(x)


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e8m0fnu, torch.uint8, torch.float4_e2m1fn_x2):
        return t.view(torch.uint8).numpy()
    if t.dtype == torch.float32:
        return t.numpy().view(np.uint32)
    return t.numpy()


def np_bits(a: np.ndarray) -> np.ndarray:
    a = np.asarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a
