"""GPU parity of the MXFP4 expert path (E2M1 + E8M0/32 weights on the
tcgen05 kind::mxf4 block32 MMA, activations fed as four MXFP4 residual terms)
against the reference's MXFP4 construction: decoded weights times unquantized
activations (layer10_moe.py:571-593, 711-738), FP32/double accumulation.

Tolerance (north star): max |gpu - oracle| / max |oracle| <= 1e-2 and cosine
similarity >= 0.9999.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from moe_fixtures import bf16_to_np, make_expert_mxfp4, oracle_forward

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MIN_COS = 0.9999


def _layer(H, I, E, k, shared, max_tokens):
    from glm5x_moe.layer import GLM5XMoELayer
    return GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=k,
                         has_shared=shared, max_tokens=max_tokens, precision="mxfp4")


def _assert_close(got, want, what):
    max_rel, l2, cos = O.relative_error(got, want)
    assert max_rel <= MAX_REL and cos >= MIN_COS, (what, max_rel, l2, cos)


@pytest.mark.parametrize("T,bn,weight_rows", [(1, 0, 128), (5, 0, 128), (40, 0, 128),
                                              (300, 0, 128), (9, 32, 128), (20, 64, 128),
                                              (40, 128, 128), (150, 256, 128),
                                              (300, 256, 128), (1, 0, 256), (9, 32, 256),
                                              (20, 64, 256), (40, 0, 256)])
def test_mxfp4_routed_expert_path(T, bn, weight_rows):
    """Every token-tile width, segments spanning several tiles, the shared
    expert, and term rows padded inside a tile."""
    H, I, E, k = 512, 512, 8, 2
    layer = _layer(H, I, E, k, True, 320)
    layer.set_tile_n(bn)
    layer.set_weight_tile_rows(weight_rows)
    deq = {}
    for e in list(range(E)) + [-1]:
        ex, dq = make_expert_mxfp4(H, I, 3000 + e)
        layer.load_expert(e, ex)
        deq[e] = dq
    rng = np.random.default_rng(100 + T)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32) + 0.25
    hidden = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16)
    out = layer.forward_routed(hidden.cuda(), torch.from_numpy(ids), torch.from_numpy(w))
    layer.check()
    shared = deq.pop(-1)
    want, _ = oracle_forward(bf16_to_np(hidden), ids, w, deq, shared,
                             expert_fn=O.mxfp4_expert_oracle)
    _assert_close(out.cpu().numpy(), want, f"T={T} bn={bn} w={weight_rows}")
    layer.close()


def test_mxfp4_glm_shape_router_decode():
    """Decode-shaped batch (64 tokens) through the router and 16 GLM-shaped
    MXFP4 experts (6144 -> 2048 -> 6144) plus the shared expert."""
    H, I, E, k, T = 6144, 2048, 16, 8, 64
    layer = _layer(H, I, E, k, True, T)
    deq = {}
    for e in list(range(E)) + [-1]:
        ex, dq = make_expert_mxfp4(H, I, 70 + e)
        layer.load_expert(e, ex)
        deq[e] = dq
    g = torch.Generator().manual_seed(77)
    router = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.rand(E, generator=g) * 0.2 - 0.1
    layer.set_router(router, bias)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
    res = layer(hidden.cuda())
    shared = deq.pop(-1)
    want, _ = oracle_forward(bf16_to_np(hidden), res.topk_indices.numpy(),
                             res.topk_weights.numpy(), deq, shared,
                             expert_fn=O.mxfp4_expert_oracle)
    _assert_close(res.output.cpu().numpy(), want, "layer")
    layer.close()


def test_mxfp4_admission_contract():
    """Host-pointer admission (the .pm4 / k3x record layout): a reserved 0xFF
    E8M0 scale is rejected with GLM5X_INVALID_MXFP4 (15) like the reference's
    decode_mxfp4; wrong group sizes and an NVFP4 engine are rejected too."""
    from glm5x_moe import _native as N
    from glm5x_moe.layer import GLM5XMoELayer
    H, I = 512, 512
    layer = _layer(H, I, 4, 2, False, 8)
    ex, _ = make_expert_mxfp4(H, I, 5)
    mats = []
    keep = []
    for q in (ex.gate_proj, ex.up_proj, ex.down_proj):
        p = q.packed.cpu().numpy().copy()
        s = q.scales.cpu().numpy().copy()
        keep += [p, s]
        mats.append(N.Mxfp4Matrix(p.ctypes.data, s.ctypes.data, q.shape[0], q.shape[1], 32))
    lib = N.lib()
    assert lib.glm5x_moe_load_expert_mxfp4(layer._h, 0, *[ctypes.byref(m) for m in mats]) == 0
    keep[3][17] = 0xFF  # up scales
    assert lib.glm5x_moe_load_expert_mxfp4(layer._h, 1, *[ctypes.byref(m) for m in mats]) == 15
    keep[3][17] = 0x7F
    bad = N.Mxfp4Matrix(mats[2].packed, mats[2].scales, H, I, 16)
    assert lib.glm5x_moe_load_expert_mxfp4(layer._h, 1, ctypes.byref(mats[0]),
                                           ctypes.byref(mats[1]), ctypes.byref(bad)) == 9
    layer.close()
    nv = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=4, top_k=2,
                       has_shared=False, max_tokens=8)
    assert lib.glm5x_moe_load_expert_mxfp4(nv._h, 0, *[ctypes.byref(m) for m in mats]) == 16
    nv.close()
