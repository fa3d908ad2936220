"""Checkpoint tensors -> the kernel-native layout of this library.

The reference streams HF safetensors shards and converts each tensor on the
fly (weight_loader.py:98-201): HF names become the model's names, routed
experts outside this rank's contiguous range are skipped, tensor-parallel
weights are sliced, int8 expert weights are reinterpreted as packed e2m1
(float4_e2m1fn_x2), and each ``wo_a`` weight is fused with its 128x128 block
scales into bf16.  This module does the same per-tensor conversion on the
device, then assembles each MoE layer's experts into
:class:`moe.MoEWeights` -- W1 and W3 stacked per expert and their ue8m0
scales re-laid out once into the tcgen05 chunk layout -- so the grouped
kernels read them in place with no per-call conversion.

Inputs are ``(name, tensor)`` pairs in HF naming, from any source:
:func:`iter_safetensors` reads them from shard files (one shard open at a
time), tests build them in memory.
"""

from __future__ import annotations

import os
import re
from glob import glob
from typing import Dict, Iterable, Iterator, Optional, Tuple

import torch

from . import _lib

__all__ = ["rename_key", "convert_tensors", "iter_safetensors", "fuse_block_scales", "moe_layer_weights",
           "local_expert_range"]

# HF module name -> (model name, tensor-parallel split dim or None).  The
# model's names and split dims are an interface of DeepSeek's model code, so
# the table lists the same pairs as weight_loader.py:51-73.
_KEYS = {
    "embed_tokens": ("embed", 0), "input_layernorm": ("attn_norm", None),
    "post_attention_layernorm": ("ffn_norm", None), "q_proj": ("wq", 0), "q_a_proj": ("wq_a", None),
    "q_a_layernorm": ("q_norm", None), "q_b_proj": ("wq_b", 0), "kv_a_proj_with_mqa": ("wkv_a", None),
    "kv_a_layernorm": ("kv_norm", None), "kv_b_proj": ("wkv_b", 0), "o_proj": ("wo", 1),
    "gate_proj": ("w1", 0), "down_proj": ("w2", 1), "up_proj": ("w3", 0), "lm_head": ("head", 0),
    "embed": ("embed", 0), "wq_b": ("wq_b", 0), "wo_a": ("wo_a", 0), "wo_b": ("wo_b", 1), "head": ("head", 0),
    "attn_sink": ("attn_sink", 0), "weights_proj": ("weights_proj", 0),
}
# names whose last component (not the module) is the key: hyper-connection
# parameters and a few per-layer vectors (weight_loader.py:85-88)
_LAST_COMPONENT_KEYS = ("hc", "attn_sink", "tie2eid", "ape")


def rename_key(name: str) -> Tuple[str, Optional[int]]:
    """HF tensor name -> (model name, tensor-parallel split dim or None)."""
    if name.startswith("model."):
        name = name[len("model."):]
    name = (name.replace("self_attn", "attn").replace("mlp", "ffn").replace("weight_scale_inv", "scale")
            .replace("e_score_correction_bias", "bias"))
    parts = name.split(".")
    key = parts[-1] if any(k in name for k in _LAST_COMPONENT_KEYS) else parts[-2]
    new_key, dim = _KEYS.get(key, (key, None))
    return name.replace(key, new_key), dim


def local_expert_range(n_experts: int, rank: int, world_size: int) -> Tuple[int, int]:
    """Contiguous routed-expert range of a rank (weight_loader.py:112-115)."""
    n = n_experts // world_size
    return rank * n, (rank + 1) * n


def _routed_expert_index(name: str) -> Optional[int]:
    if "experts" not in name or "shared_experts" in name:
        return None
    m = re.search(r"\.experts\.(\d+)\.", name)
    return int(m.group(1)) if m else None


def fuse_block_scales(weight: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """e4m3 weight [N, K] times its [ceil(N/128), K/128] block scales (fp32 or
    e8m0) -> bf16 [N, K] on the device (the ``wo_a`` fusion,
    weight_loader.py:146-163)."""
    if not weight.is_cuda:
        raise RuntimeError("fuse_block_scales runs on CUDA tensors only (no CPU fallback)")
    w = weight.contiguous().view(torch.uint8)
    N, K = w.shape
    if scale.dtype == torch.float8_e8m0fnu:
        s, sdt = scale.contiguous().view(torch.uint8), _lib.DT_E8M0
    else:
        s, sdt = scale.float().contiguous(), _lib.DT_F32
    if s.shape != ((N + 127) // 128, K // 128):
        raise ValueError(f"wo_a scale shape {tuple(s.shape)} does not match weight {tuple(w.shape)}")
    out = torch.empty(N, K, dtype=torch.bfloat16, device=weight.device)
    _lib.check(_lib.load().bs_e4m3_blocks_to_bf16(w.data_ptr(), s.data_ptr(), sdt, N, K, out.data_ptr(),
                                                  torch.cuda.current_stream(weight.device).cuda_stream))
    return out


def convert_tensors(tensors: Iterable[Tuple[str, torch.Tensor]], rank: int = 0, world_size: int = 1,
                    n_experts: int = 256, device="cuda") -> Iterator[Tuple[str, torch.Tensor]]:
    """Per-tensor conversion of HF-named tensors (weight_loader.py:122-201):
    rename, skip other ranks' routed experts and MTP embedding / head copies,
    slice tensor-parallel weights (not routed experts: they are sharded by
    expert range), view int8 expert weights as packed e2m1,
    fuse each ``wo_a`` weight with its scale into bf16.  Yields
    (model name, tensor on `device`)."""
    e_lo, e_hi = local_expert_range(n_experts, rank, world_size)
    pending: Dict[str, torch.Tensor] = {}
    for orig, t in tensors:
        if orig.startswith("model.mtp.") and ("emb" in orig or orig.endswith("head.weight")):
            continue
        name, dim = rename_key(orig)
        e = _routed_expert_index(name)
        if e is not None and not (e_lo <= e < e_hi):
            continue
        # routed experts are sharded by expert range only and stay whole (the
        # expert-parallel layer needs whole experts); the reference's loader
        # also narrows their w1/w2/w3 along the tensor-parallel dim
        if dim is not None and world_size > 1 and e is None:
            size = t.size(dim) // world_size
            t = t.narrow(dim, rank * size, size).contiguous()
        if name.endswith("wo_a.weight") or name.endswith("wo_a.scale"):
            pending[name] = t
            w_name = name[:-len("scale")] + "weight" if name.endswith("scale") else name
            s_name = w_name[:-len("weight")] + "scale"
            if w_name in pending and s_name in pending:
                yield w_name, fuse_block_scales(pending.pop(w_name).to(device), pending.pop(s_name).to(device))
            continue
        if e is not None and t.dtype == torch.int8:
            t = t.view(torch.float4_e2m1fn_x2)
        yield name, t.to(device)
    for name, t in pending.items():      # a wo_a part whose partner never came
        yield name, t.to(device)


def iter_safetensors(path: str) -> Iterator[Tuple[str, torch.Tensor]]:
    """(HF name, tensor) pairs from the ``*.safetensors`` shards of a
    checkpoint directory, one shard open at a time."""
    from safetensors import safe_open
    files = sorted(glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {path}")
    for fn in files:
        with safe_open(fn, framework="pt", device="cpu") as f:
            for k in f.keys():
                yield k, f.get_tensor(k)


def moe_layer_weights(converted: Dict[str, torch.Tensor], layer: int, n_experts: int, rank: int = 0,
                      world_size: int = 1):
    """One MoE layer's routed experts of this rank, from converted tensors
    (``layers.{layer}.ffn.experts.{e}.{w1,w2,w3}.{weight,scale}``), in the
    kernel-native form: W1|W3 stacked [El, 2I, H/2], W2 [El, H, I/2], ue8m0
    scales packed once into the tcgen05 chunk layout."""
    from .moe import MoEWeights
    e_lo, e_hi = local_expert_range(n_experts, rank, world_size)
    pre = f"layers.{layer}.ffn.experts."

    def get(e, w, what):
        t = converted[f"{pre}{e}.{w}.{what}"]
        return t.view(torch.uint8) if what == "weight" else t

    w13 = torch.stack([torch.cat([get(e, "w1", "weight"), get(e, "w3", "weight")]) for e in range(e_lo, e_hi)])
    w13_s = torch.stack([torch.cat([get(e, "w1", "scale"), get(e, "w3", "scale")]) for e in range(e_lo, e_hi)])
    w2 = torch.stack([get(e, "w2", "weight") for e in range(e_lo, e_hi)])
    w2_s = torch.stack([get(e, "w2", "scale") for e in range(e_lo, e_hi)])
    if w13_s.dtype != torch.float8_e8m0fnu or w2_s.dtype != torch.float8_e8m0fnu:
        raise TypeError("expert weight scales must be float8_e8m0fnu (the checkpoints' ue8m0 1x32 scales)")
    return MoEWeights(w13, w13_s.view(torch.uint8), w2, w2_s.view(torch.uint8))
