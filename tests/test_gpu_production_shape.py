"""GPU parity at the production shape: hidden 6144, intermediate 2048, 256
routed experts + 1 shared, top-8, routed scaling 2.5 (configs C3, C4, C5).

- The tcgen05 router at T = 1024 (the contraction split along K over several
  CTAs, partial logits summed in fixed order) and T = 8192 (two K planes)
  against the oracle's sequential FP32 router (layer10_moe.py:760-789 /
  select_routing, routing_policy.cpp:31-159): ids equal except where the
  k-th and (k+1)-th choice scores are within 1e-5 of each other; weights
  within 1e-5 relative where the ids agree.
- C3: the whole NVFP4 layer at T = 1024 over all 257 segments, every token
  against the FP32 dequant-matmul oracle (per-slab re-quantized activations,
  layer10_moe.py:711-738, nvfp4.py:294-335).
- C4: the whole MXFP4 layer at decode batch 64 with the Zipf-skewed router,
  the full batch against the MXFP4 oracle (decoded weights x unquantized
  activations, layer10_moe.py:571-593).

Tolerance (north star): max |gpu - oracle| / max |oracle| <= 1e-2 and cosine
similarity >= 0.9999. The oracle dequantizes one expert at a time so the
host never holds all 257 experts in FP32.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from moe_fixtures import bf16_to_np, oracle_forward

pytestmark = pytest.mark.gpu

H, I, E, K_TOP, SCALE = 6144, 2048, 256, 8, 2.5
MAX_REL = 1e-2
MIN_COS = 0.9999
NEAR_TIE = 1e-5


def _assert_close(got, want, what):
    max_rel, l2, cos = O.relative_error(got, want)
    assert max_rel <= MAX_REL and cos >= MIN_COS, (what, max_rel, l2, cos)


def _router(seed: int, zipf: bool = False):
    g = torch.Generator().manual_seed(seed)
    router = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    bias = torch.rand(E, generator=g) * 0.2 - 0.1
    if zipf:  # config 4: bias_e += 0.5 * (pi(e) + 1)^-1.1 for a seeded permutation pi
        perm = torch.randperm(E, generator=g)
        bias = bias + 0.5 * (perm.to(torch.float64) + 1.0).pow(-1.1).to(torch.float32)
    return router, bias


def _hidden(T: int, seed: int) -> torch.Tensor:
    """Config-5 style hidden states: drafts of one sequence share a base row."""
    g = torch.Generator().manual_seed(seed)
    seqs = max(T // 4, 1)
    base = torch.randn(seqs, 1, H, generator=g)
    eps = torch.randn(seqs, T // seqs, H, generator=g)
    h = (base + 0.25 * eps).reshape(-1, H)[:T]
    h = h / h.pow(2).mean(dim=1, keepdim=True).sqrt()
    return h.to(torch.bfloat16)


def _check_routes(x, router, bias, ids_g, w_g, logits_g=None):
    """ids_g / w_g [n, k] from the device for token rows x [n, H]: identical
    to the oracle's except at near-ties of the k-th and (k+1)-th choice."""
    ids_o, w_o, logits_o = O.route_tokens(x, router.float().numpy(), bias.numpy(), K_TOP, SCALE,
                                          want_logits=True)
    if logits_g is not None:
        assert np.abs(logits_g - logits_o).max() < 1e-3
    ties = 0
    b = bias.numpy().astype(np.float64)
    for t in range(x.shape[0]):
        if np.array_equal(ids_g[t], ids_o[t]):
            np.testing.assert_allclose(w_g[t], w_o[t], rtol=1e-5, atol=0, err_msg=str(t))
            continue
        sc = 1.0 / (1.0 + np.exp(-logits_o[t].astype(np.float64))) + b
        kth = np.sort(sc)[::-1][K_TOP - 1:K_TOP + 1]
        assert kth[0] - kth[1] <= NEAR_TIE, (t, ids_g[t], ids_o[t], kth)
        # the selected sets may only differ in the tied k-th place
        assert len(set(ids_g[t]) ^ set(ids_o[t])) <= 2, t
        ties += 1
    return ties


def _gpu_experts(seed: int, precision: str, dev):
    """Seeded GLM-shaped experts (N(0, 0.02) BF16 weights generated on the
    device) packed by the library's GPU packer; 256 routed + shared (-1)."""
    from glm5x_moe.layer import MXFP4Expert, NVFP4Expert
    from glm5x_moe.nvfp4 import quantize_mxfp4_weight, quantize_nvfp4_weight
    g = torch.Generator(device=dev).manual_seed(seed)
    out = {}
    for e in list(range(E)) + [-1]:
        mats = []
        for shape in ((I, H), (I, H), (H, I)):
            w = (torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            mats.append(quantize_nvfp4_weight(w, scale_mode="mse") if precision == "nvfp4"
                        else quantize_mxfp4_weight(w))
        out[e] = NVFP4Expert(*mats) if precision == "nvfp4" else MXFP4Expert(*mats)
    return out


class _LazyDequant(dict):
    """experts_deq for oracle_forward that dequantizes an expert (oracle C
    code) only when it is looked up, and keeps nothing."""

    def __init__(self, experts, precision):
        super().__init__()
        self._experts, self._precision = experts, precision

    def __getitem__(self, e):
        ex = self._experts[e]
        deq = []
        for q, shape in ((ex.gate_proj, (I, H)), (ex.up_proj, (I, H)), (ex.down_proj, (H, I))):
            if self._precision == "nvfp4":
                deq.append(O.nvfp4_dequantize(q.packed.cpu().numpy(), q.scale_bytes().cpu().numpy(),
                                              float(q.global_scale.item()), *shape))
            else:
                deq.append(O.mxfp4_decode(q.packed.cpu().numpy(), q.scales.cpu().numpy(), *shape))
        return tuple(deq)


@pytest.mark.parametrize("T", [1024, 8192])
def test_router_256_experts_split_k(T):
    """The tcgen05 router over 256 experts: T = 1024 splits the K = 6144
    contraction over many CTAs per 128-token tile (fixed-order partial sums,
    then the top-k kernel); T = 8192 runs two K planes. Checked on a sample
    of 1024 tokens spread over every 128-token tile."""
    from glm5x_moe.layer import GLM5XMoELayer
    layer = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=K_TOP,
                          routed_scaling_factor=SCALE, has_shared=True, max_tokens=T)
    router, bias = _router(11 + T)
    layer.set_router(router, bias)
    hidden = _hidden(T, 5 + T)
    ids, w = layer.route(hidden.cuda())
    torch.cuda.synchronize()
    layer.check()
    ids_g, w_g = ids.cpu().numpy(), w.cpu().numpy()
    sample = np.arange(T) if T <= 1024 else np.sort(
        np.random.default_rng(T).choice(T, 1024, replace=False))
    x = bf16_to_np(hidden)[sample]
    ties = _check_routes(x, router, bias, ids_g[sample], w_g[sample])
    assert ties <= len(sample) // 100, ties
    layer.close()


def test_c3_full_layer_256_experts():
    """Config 3: T = 1024 through the router and every one of the 257 NVFP4
    segments (256 routed + shared, 256-row token tiles on CTA pairs), each
    token's output against the per-slab FP32 dequant-matmul oracle."""
    from glm5x_moe.layer import GLM5XMoELayer
    T = 1024
    dev = torch.device("cuda", 0)
    layer = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=K_TOP,
                          routed_scaling_factor=SCALE, has_shared=True, max_tokens=T)
    experts = _gpu_experts(3, "nvfp4", dev)
    for e, ex in experts.items():
        layer.load_expert(e, ex)
    router, bias = _router(1)
    layer.set_router(router, bias)
    hidden = _hidden(T, 2)
    res = layer(hidden.cuda())
    x = bf16_to_np(hidden)
    ids_g, w_g = res.topk_indices.numpy(), res.topk_weights.numpy()
    _check_routes(x, router, bias, ids_g, w_g, res.router_logits.numpy())
    assert len(np.unique(ids_g)) > 150  # the grid really spans the experts
    deq = _LazyDequant(experts, "nvfp4")
    want, _ = oracle_forward(x, ids_g, w_g, deq, deq[-1])
    _assert_close(res.output.cpu().numpy(), want, "c3 layer")
    layer.close()


def test_c4_mxfp4_decode_256_experts():
    """Config 4 on one GPU: decode batch 64, 256 MXFP4 experts + shared, the
    Zipf(1.1)-skewed router bias; the whole batch against the MXFP4 oracle."""
    from glm5x_moe.layer import GLM5XMoELayer
    T = 64
    dev = torch.device("cuda", 0)
    layer = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=K_TOP,
                          routed_scaling_factor=SCALE, has_shared=True, max_tokens=T,
                          precision="mxfp4")
    experts = _gpu_experts(4, "mxfp4", dev)
    for e, ex in experts.items():
        layer.load_expert(e, ex)
    router, bias = _router(5, zipf=True)
    layer.set_router(router, bias)
    hidden = torch.randn(T, H, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16)
    res = layer(hidden.cuda())
    x = bf16_to_np(hidden)
    ids_g, w_g = res.topk_indices.numpy(), res.topk_weights.numpy()
    _check_routes(x, router, bias, ids_g, w_g, res.router_logits.numpy())
    deq = _LazyDequant(experts, "mxfp4")
    want, _ = oracle_forward(x, ids_g, w_g, deq, deq[-1], expert_fn=O.mxfp4_expert_oracle)
    _assert_close(res.output.cpu().numpy(), want, "c4 decode")
    layer.close()
