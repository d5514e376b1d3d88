"""The per-token max |x| that the NVFP4 slab scales start from is taken by the
tensor-core router from the token tiles it streams (one K plane per CTA, or
several planes meeting in an atomic max), instead of a separate pass over the
batch. The forward that routes itself must therefore give exactly the output
of the expert path run on the same routing with the stand-alone row-amax
kernel (glm5x_moe_forward_routed), bit for bit: both K-split (small batches)
and unsplit (more token tiles than half the SMs) routers, and rows whose
largest value sits in any 64-column K step.
"""
from __future__ import annotations

import pytest
import torch

from moe_fixtures import make_expert

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [24, 300, 9600])
def test_router_amax_matches_row_amax_kernel(T):
    from glm5x_moe.layer import GLM5XMoELayer
    H, I, E, k = 512, 512, 16, 4
    layer = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=k,
                          has_shared=True, max_tokens=T, device=0)
    for e in list(range(E)) + [-1]:
        ex, _ = make_expert(H, I, 4000 + e)
        layer.load_expert(e, ex)
    g = torch.Generator().manual_seed(T)
    router = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.rand(E, generator=g) * 0.2 - 0.1
    layer.set_router(router, bias)
    hidden = torch.randn(T, H, generator=g)
    # each row's largest |x| in a different K step, some negative
    cols = torch.randint(0, H, (T,), generator=g)
    spikes = (torch.rand(T, generator=g) * 20 + 5) * torch.where(torch.rand(T, generator=g) < 0.5,
                                                               -1.0, 1.0)
    hidden[torch.arange(T), cols] = spikes
    hidden = hidden.to(torch.bfloat16).cuda()
    res = layer(hidden)
    layer.check()
    again = layer.forward_routed(hidden, res.topk_indices.cuda(), res.topk_weights.cuda())
    layer.check()
    assert torch.equal(res.output.cpu(), again.cpu())
    layer.close()
