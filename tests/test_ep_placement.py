"""Expert placement for expert parallelism from the router's correction bias
(glm5x_moe.ep.bias_balanced_order): a permutation that gives every rank
E / W experts of every bias level, and on config 5's synthetic routing
(router N(0, 0.02), bias U(-0.1, 0.1), MTP-draft hidden states) an even
spread of routed rows over the ranks, which contiguous expert-id ranges do
not give."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from glm5x_moe.ep import bias_balanced_order, expert_range


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_permutation_and_snake(world):
    rng = np.random.default_rng(world)
    bias = rng.random(256) * 0.2 - 0.1
    order = bias_balanced_order(bias, world)
    assert sorted(order) == list(range(256))
    per = 256 // world
    ranked = sorted(range(256), key=lambda e: (-bias[e], e))
    for r in range(world):
        begin, count = expert_range(r, world, 256)
        assert (begin, count) == (r * per, per)
        held = set(order[begin:begin + count])
        # one expert from every round of `world` bias-ranked experts
        for rnd in range(per):
            assert len(held & set(ranked[rnd * world:(rnd + 1) * world])) == 1


def test_uneven_world_refused():
    with pytest.raises(ValueError):
        bias_balanced_order([0.0] * 10, 4)


def test_config5_rows_even_out():
    """Routed rows per rank at 4 ranks of 1024 tokens each (a reduced config
    5 batch, the same router construction as bench.py)."""
    H, E, W, T = 6144, 256, 4, 1024
    gc = torch.Generator().manual_seed(1)
    router = (torch.randn(E, H, generator=gc) * 0.02).to(torch.bfloat16).float()
    bias = torch.rand(E, generator=gc) * 0.2 - 0.1
    counts = np.zeros(E, dtype=np.int64)
    for r in range(W):
        g = torch.Generator().manual_seed(100 + r)
        base = torch.randn(T // 4, 1, H, generator=g)
        h = (base + 0.25 * torch.randn(T // 4, 4, H, generator=g)).reshape(-1, H)
        h = (h / h.pow(2).mean(dim=1, keepdim=True).sqrt()).to(torch.bfloat16).float()
        ids = (torch.sigmoid(h @ router.T) + bias).topk(8, dim=1).indices
        counts += np.bincount(ids.flatten().numpy(), minlength=E)
    order = np.array(bias_balanced_order(bias.numpy(), W))
    placed = counts[order].reshape(W, -1).sum(1)
    contiguous = counts.reshape(W, -1).sum(1)
    assert placed.max() / placed.mean() < 1.05, placed
    assert contiguous.max() / contiguous.mean() > placed.max() / placed.mean(), contiguous
