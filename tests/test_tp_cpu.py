"""Host logic of the tensor-parallel GEMM: the column split and the weight
shards each rank takes (no GPU needed)."""

from __future__ import annotations

import importlib

import pytest
import torch

from conftest import PKG_NAME


def tp():
    return importlib.import_module(PKG_NAME + ".tp")


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_column_ranges_tile_N(world):
    N = 4096
    ranges = [tp().column_range(N, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == N
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    assert all((c1 - c0) % 128 == 0 for c0, c1 in ranges)


def test_column_range_rejects_unaligned_split():
    with pytest.raises(ValueError):
        tp().column_range(4096 + 128, 2, 0)
    with pytest.raises(ValueError):
        tp().column_range(1024, 16, 0)


@pytest.mark.parametrize("fp4", [False, True])
def test_shards_reassemble_the_weight(fp4):
    N, K, world = 1024, 512, 4
    g = torch.Generator().manual_seed(3)
    if fp4:
        b = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8)
        b_s = torch.randint(120, 128, (N, K // 32), generator=g, dtype=torch.uint8)
    else:
        b = torch.randint(0, 120, (N, K), generator=g, dtype=torch.uint8)
        b_s = torch.rand(N // 128, K // 128, generator=g)
    parts = [tp().shard_weight(b, b_s, world, r, fp4) for r in range(world)]
    assert torch.equal(torch.cat([p[0] for p in parts]), b)
    assert torch.equal(torch.cat([p[1] for p in parts]), b_s)
    for pb, ps in parts:
        assert pb.is_contiguous() and ps.is_contiguous()
