"""BF16 expert admission (glm5x_moe_load_expert_bf16): float experts packed
on the device when they are loaded, as the reference's NVFP4 mode packs them
(_quantize_expert_nvfp4, layer10_moe.py:603-619 -> quantize_nvfp4_weight,
scale_mode "mse"). The resident weights must be those of loading the packed
expert (whose packer is pinned to the reference's bytes in
test_gpu_kernels.py), so the layer outputs are compared bit for bit, and the
layer itself against the FP32 dequant-matmul oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from moe_fixtures import bf16_to_np, oracle_forward

pytestmark = pytest.mark.gpu


def _bf16_expert(H, I, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(shape, generator=g) * 0.02).to(torch.bfloat16)
            for shape in ((I, H), (I, H), (H, I))]


@pytest.mark.parametrize("precision,H,I,E,k,T,on_device",
                         [("nvfp4", 512, 1024, 16, 2, 48, False),
                          ("nvfp4", 512, 1024, 16, 2, 48, True),
                          ("mxfp4", 512, 1024, 16, 2, 48, False),
                          ("nvfp4", 6144, 2048, 16, 1, 16, False)])
def test_bf16_admission_equals_packed_admission(precision, H, I, E, k, T, on_device):
    from glm5x_moe.layer import GLM5XMoELayer, MXFP4Expert, NVFP4Expert
    from glm5x_moe.nvfp4 import quantize_mxfp4_weight, quantize_nvfp4_weight
    make = lambda: GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=k,
                                 has_shared=True, max_tokens=T, precision=precision)
    a, b = make(), make()
    deq = {}
    for e in list(range(E)) + [-1]:
        w = _bf16_expert(H, I, 40 + e)
        a.load_expert_bf16(e, *[t.cuda() if on_device else t for t in w],
                           scale_mode="mse" if precision == "nvfp4" else "max_abs")
        if precision == "nvfp4":
            q = [quantize_nvfp4_weight(t.cuda(), scale_mode="mse") for t in w]
            b.load_expert(e, NVFP4Expert(*q))
            deq[e] = tuple(O.nvfp4_dequantize(m.packed.cpu().numpy(), m.scale_bytes().cpu().numpy(),
                                              float(m.global_scale.item()), *t.shape)
                           for m, t in zip(q, w))
        else:
            q = [quantize_mxfp4_weight(t.cuda()) for t in w]
            b.load_expert(e, MXFP4Expert(*q))
            deq[e] = tuple(O.mxfp4_decode(m.packed.cpu().numpy(), m.scales.cpu().numpy(), *t.shape)
                           for m, t in zip(q, w))
    g = torch.Generator().manual_seed(5)
    router = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.rand(E, generator=g) * 0.2 - 0.1
    for layer in (a, b):
        layer.set_router(router, bias)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
    ra, rb = a(hidden.cuda()), b(hidden.cuda())
    assert torch.equal(ra.topk_indices, rb.topk_indices)
    assert torch.equal(ra.output, rb.output)
    shared = deq.pop(-1)
    fn = O.nvfp4_expert_dequant_oracle if precision == "nvfp4" else O.mxfp4_expert_oracle
    want, _ = oracle_forward(bf16_to_np(hidden), ra.topk_indices.numpy(),
                             ra.topk_weights.numpy(), deq, shared, expert_fn=fn)
    max_rel, _, cos = O.relative_error(ra.output.cpu().numpy(), want)
    assert max_rel <= 1e-2 and cos >= 0.9999, (max_rel, cos)
    a.close()
    b.close()


def test_bf16_admission_rejects_bad_arguments():
    from glm5x_moe._native import Glm5xError
    from glm5x_moe.layer import GLM5XMoELayer
    layer = GLM5XMoELayer(hidden_size=512, intermediate_size=1024, num_experts=4, top_k=2,
                          has_shared=False, max_tokens=8)
    w = _bf16_expert(512, 1024, 1)
    with pytest.raises(ValueError, match="SHAPE"):
        layer.load_expert_bf16(0, w[2], w[1], w[0])
    with pytest.raises(Glm5xError, match="not held"):
        layer.load_expert_bf16(7, *w)
    bad = w[0].clone()
    bad[3, 5] = float("inf")
    with pytest.raises(Glm5xError, match="non-finite"):
        layer.load_expert_bf16(0, bad, w[1], w[2])
    layer.close()
