"""Checkpoint conversion (loader.py) on synthetic HF-named tensors: names,
the routed-expert range filter, tensor-parallel slicing, the int8 -> packed
e2m1 view (CPU); the wo_a fusion and the assembled MoE weights against the
numpy restatement and the unconverted layer (GPU)."""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from conftest import PKG_NAME
from oracle import blockscaled as ob


def loader():
    return importlib.import_module(PKG_NAME + ".loader")


def _ckpt(E=8, H=256, I=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    t = {}
    for e in range(E):
        for hf, rows, k in (("gate_proj", I, H), ("up_proj", I, H), ("down_proj", H, I)):
            t[f"model.layers.3.mlp.experts.{e}.{hf}.weight"] = torch.randint(-128, 128, (rows, k // 2), generator=g,
                                                                              dtype=torch.int8)
            t[f"model.layers.3.mlp.experts.{e}.{hf}.weight_scale_inv"] = (
                127 - torch.randint(0, 7, (rows, k // 32), generator=g, dtype=torch.uint8)).view(torch.float8_e8m0fnu)
    t["model.layers.3.mlp.shared_experts.gate_proj.weight"] = torch.randn(2 * I, H, generator=g).to(torch.bfloat16)
    t["model.layers.3.self_attn.wo_a.weight"] = (torch.randn(256, 384, generator=g) * 40).clamp(-448, 448).to(
        torch.float8_e4m3fn)
    t["model.layers.3.self_attn.wo_a.weight_scale_inv"] = torch.rand(2, 3, generator=g) + 0.01
    t["model.layers.3.input_layernorm.weight"] = torch.ones(H)
    t["model.mtp.0.emb.weight"] = torch.zeros(4, H)
    return t


def test_rename_key():
    L = loader()
    assert L.rename_key("model.layers.0.mlp.experts.7.gate_proj.weight") == ("layers.0.ffn.experts.7.w1.weight", 0)
    assert L.rename_key("model.layers.0.mlp.experts.7.down_proj.weight_scale_inv") == \
        ("layers.0.ffn.experts.7.w2.scale", 1)
    assert L.rename_key("model.layers.1.self_attn.q_b_proj.weight") == ("layers.1.attn.wq_b.weight", 0)
    assert L.rename_key("model.layers.1.input_layernorm.weight") == ("layers.1.attn_norm.weight", None)
    assert L.rename_key("model.layers.1.mlp.gate.e_score_correction_bias") == ("layers.1.ffn.gate.bias", None)


@pytest.mark.parametrize("rank,world", [(0, 1), (1, 2), (3, 4)])
def test_convert_filters_experts_and_slices(rank, world):
    L = loader()
    ck = {k: v for k, v in _ckpt().items() if "wo_a" not in k}
    out = dict(L.convert_tensors(ck.items(), rank=rank, world_size=world, n_experts=8, device="cpu"))
    lo, hi = L.local_expert_range(8, rank, world)
    experts = sorted({int(k.split(".")[4]) for k in out if ".experts." in k})
    assert experts == list(range(lo, hi))
    w = out[f"layers.3.ffn.experts.{lo}.w1.weight"]
    assert w.dtype == torch.float4_e2m1fn_x2 and tuple(w.shape) == (128, 128)     # whole expert, packed e2m1
    assert torch.equal(w.view(torch.uint8), ck[f"model.layers.3.mlp.experts.{lo}.gate_proj.weight"].view(torch.uint8))
    sh = out["layers.3.ffn.shared_experts.w1.weight"]
    assert sh.shape[0] == 256 // world                                          # tensor-parallel slice
    assert not any("mtp" in k for k in out)


@pytest.mark.gpu
def test_wo_a_fusion_matches_numpy():
    L = loader()
    ck = _ckpt()
    out = dict(L.convert_tensors(ck.items(), n_experts=8))
    got = out["layers.3.attn.wo_a.weight"]
    assert got.dtype == torch.bfloat16 and tuple(got.shape) == (256, 384)
    w = ob.e4m3_to_f32(ck["model.layers.3.self_attn.wo_a.weight"].view(torch.uint8).numpy())
    s = ck["model.layers.3.self_attn.wo_a.weight_scale_inv"].numpy()
    ref = ob.f32_to_bf16((w.reshape(2, 128, 3, 128) * s[:, None, :, None]).reshape(256, 384).astype(np.float32))
    np.testing.assert_array_equal(got.cpu().view(torch.int16).numpy().view(np.uint16), ref)


@pytest.mark.gpu
def test_moe_layer_weights_match_direct_construction():
    L = loader()
    mm = importlib.import_module(PKG_NAME + ".moe")
    ck = _ckpt()
    conv = dict(L.convert_tensors(ck.items(), n_experts=8))
    W = L.moe_layer_weights(conv, 3, 8)
    raw = lambda e, hf, s="weight": ck[f"model.layers.3.mlp.experts.{e}.{hf}.{s}"].view(torch.uint8)   # noqa: E731
    w13 = torch.stack([torch.cat([raw(e, "gate_proj"), raw(e, "up_proj")]) for e in range(8)]).cuda()
    w13_s = torch.stack([torch.cat([raw(e, "gate_proj", "weight_scale_inv"), raw(e, "up_proj", "weight_scale_inv")])
                         for e in range(8)]).cuda()
    w2 = torch.stack([raw(e, "down_proj") for e in range(8)]).cuda()
    w2_s = torch.stack([raw(e, "down_proj", "weight_scale_inv") for e in range(8)]).cuda()
    ref = mm.MoEWeights(w13, w13_s, w2, w2_s)
    assert (W.E, W.H, W.I) == (8, 256, 128)
    for a in ("w13", "w13_sp", "w2", "w2_sp"):
        assert torch.equal(getattr(W, a), getattr(ref, a)), a
