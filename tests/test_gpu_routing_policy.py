"""GPU routing policy: the batched select_routing (glm5x_select_routing_policy)
against the oracle restatement token by token, and the engine with a fixed /
adaptive policy end to end (router -> reduced routes -> experts) against the
oracle's decisions and expert math.

Bars: expert ids, selected K, escalation and the routing weights bit-exact
(the same FP32 operations); entropy, effective support, mass and confidence
within 1e-6 relative or absolute (device logf / expf against the host's). Layer outputs: max rel
err <= 1e-2 and cosine >= 0.9999 as for every expert path.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from moe_fixtures import bf16_to_np, make_expert, oracle_forward

pytestmark = pytest.mark.gpu

CONFIGS = [("natural", dict(), 8), ("natural", dict(), 16), ("fixed", dict(fixed_k=4), 8),
           ("fixed", dict(fixed_k=12), 16), ("fixed", dict(fixed_k=6, quality_floor_k=8), 16),
           ("adaptive", dict(), 16), ("adaptive", dict(mass_target=0.6,
                                                       minimum_boundary_gap=0.05), 16),
           ("adaptive", dict(mass_target=0.5, quality_floor_k=8), 16),
           ("adaptive", dict(mass_target=1.0), 16)]


def _scores(T, E, seed):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(T, E, generator=g) * 2.0
    peaked = torch.rand(T, generator=g) < 0.3
    logits[peaked, :6] += 6.0  # a few dominant experts on some tokens
    scores = torch.sigmoid(logits).float()
    bias = (torch.rand(E, generator=g) * 0.2 - 0.1).float()
    return scores, bias


LADDER = (4, 6, 8, 12, 16)
EPS = 1e-5  # routing_policy.cpp:13 comparison_epsilon


def _near_tie(scores, bias, natural_k, cfg, k_gpu, k_orc, tol=1e-5):
    """True when the decision of select_routing (routing_policy.cpp:31-159)
    for these scores sits within `tol` of a boundary, computed in double:
    two choice scores adjacent in the natural order up to position
    natural_k + 1 within `tol`, or, for a ladder K between the two selected
    K, a mass / effective-support / boundary-gap test within `tol` of its
    threshold. Only such tokens may decide differently on the device."""
    s = np.asarray(scores, dtype=np.float64)
    c = s + np.asarray(bias, dtype=np.float64)
    order = np.argsort(-c, kind="stable")
    cs = c[order[:natural_k + 1]]
    if np.any(cs[:-1] - cs[1:] <= tol):
        return True
    if k_gpu == k_orc:
        return False
    p = s[order[:natural_k]] / s[order[:natural_k]].sum()
    ent = -np.sum(p[p > 0] * np.log(p[p > 0]))
    support = np.exp(ent)
    lo, hi = min(k_gpu, k_orc), max(k_gpu, k_orc)
    for K in LADDER:
        if not lo <= K <= hi or K > natural_k:
            continue
        mass = p[:K].sum()
        gap = 1.0 if K >= natural_k else max(p[K - 1] - p[K], 0.0) / p[0]
        if (abs(mass + EPS - cfg.mass_target) <= tol or abs(K + EPS - support) <= tol
                or abs(gap + EPS - cfg.minimum_boundary_gap) <= tol):
            return True
    return False


@pytest.mark.parametrize("mode,kw,k", CONFIGS)
def test_batched_select_routing(mode, kw, k):
    from glm5x_moe.routing import RoutingMode, RoutingPolicyConfig, select_routing
    T, E = 1024, 256
    scores, bias = _scores(T, E, 11 + k)
    cfg = RoutingPolicyConfig(RoutingMode(mode), **kw)
    d = select_routing(scores.cuda(), bias.cuda(), k, cfg)
    ids = d.expert_ids.cpu().numpy()
    w = d.normalized_weights.cpu().numpy()
    sel = d.selected_k.cpu().numpy()
    esc = d.quality_floor_escalated.cpu().numpy()
    diag = torch.stack([d.normalized_entropy, d.entropy_effective_support,
                        d.selected_cumulative_mass, d.boundary_confidence], 1).cpu().numpy()
    s_np, b_np = scores.numpy(), bias.numpy()
    for t in range(T):
        oi, ow, ok, oe, od = O.select_routing_policy(s_np[t], b_np, k, mode, **kw)
        assert np.array_equal(ids[t], oi), (t, ids[t], oi)
        assert np.array_equal(w[t], ow), (t, w[t], ow)
        assert sel[t] == ok and bool(esc[t]) == oe, t
        assert np.allclose(diag[t], od, rtol=1e-6, atol=1e-6), (t, diag[t], od)


def test_engine_policy_routes_and_outputs():
    """Adaptive Top-K over a natural Top-16, then fixed K = 4, through the
    whole layer: routes match the oracle's decisions on the engine's own
    logits, empty slots are skipped, outputs match the expert oracle."""
    from glm5x_moe.layer import GLM5XMoELayer
    from glm5x_moe.routing import RoutingMode, RoutingPolicyConfig
    H, I, E, k, T = 512, 512, 32, 16, 96
    layer = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=k,
                          has_shared=True, max_tokens=T)
    deq = {}
    for e in list(range(E)) + [-1]:
        ex, dq = make_expert(H, I, 900 + e)
        layer.load_expert(e, ex)
        deq[e] = dq
    g = torch.Generator().manual_seed(33)
    router = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.rand(E, generator=g) * 0.2 - 0.1
    layer.set_router(router, bias)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
    shared = deq.pop(-1)
    for cfg in (RoutingPolicyConfig(RoutingMode.ADAPTIVE, mass_target=0.7),
                RoutingPolicyConfig(RoutingMode.FIXED, fixed_k=4)):
        layer.set_routing_policy(cfg)
        res = layer(hidden.cuda())
        ids, w = res.topk_indices.numpy(), res.topk_weights.numpy()
        logits = res.router_logits.numpy()
        sel, diag = layer.routing_decisions(T)
        for t in range(T):
            s = (1.0 / (1.0 + np.exp(-logits[t].astype(np.float64)))).astype(np.float32)
            oi, ow, ok, _, _ = O.select_routing_policy(s, bias.numpy(), k, cfg.mode.value,
                                                       fixed_k=cfg.fixed_k,
                                                       mass_target=cfg.mass_target)
            kk = int(sel[t, 0])
            assert (ids[t, kk:] == -1).all() and (w[t, kk:] == 0).all(), t
            if ok == kk and np.array_equal(oi[:kk], ids[t, :kk]):
                assert np.allclose(ow[:kk] * 2.5, w[t, :kk], rtol=1e-5), t
            else:
                # the device's sigmoid may differ from this host one by an ulp,
                # which may only flip a decision that sits on a near-tie
                assert _near_tie(s, bias.numpy(), k, cfg, kk, ok), (cfg, t, kk, ok)
        stats = layer.routing_stats()
        assert stats["decisions"] == T and stats["selected_experts"] == int(sel[:, 0].sum())
        if cfg.mode is RoutingMode.FIXED:
            assert (sel[:, 0] == 4).all()
        want, _ = oracle_forward(bf16_to_np(hidden), ids, w, deq, shared)
        max_rel, _, cos = O.relative_error(res.output.cpu().numpy(), want)
        assert max_rel <= 1e-2 and cos >= 0.9999, (cfg, max_rel, cos)
    from glm5x_moe._native import Glm5xError
    with pytest.raises(Glm5xError, match="natural Top-16"):
        small = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=8,
                              has_shared=False, max_tokens=8)
        try:
            small.set_routing_policy(RoutingPolicyConfig(RoutingMode.ADAPTIVE))
        finally:
            small.close()
    layer.close()
