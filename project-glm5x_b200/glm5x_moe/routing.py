"""Routing policy of the reference's select_routing, batched on the GPU.

Mirrors k3x_ref.routing_policy (reference/k3x_ref/routing_policy.py:11-40) and
the C++ runtime (runtime/include/k3x/routing_policy.hpp:11-39,
runtime/src/routing_policy.cpp:31-159): natural Top-K, fixed K from the ladder
4/6/8/12/16, and adaptive K over a natural Top-16 (the first ladder K whose
probability mass reaches ``mass_target``, that covers the entropy's effective
support and whose boundary gap reaches ``minimum_boundary_gap``), with an
optional quality floor. Decisions for every token are made by the engine's
top-k kernel; slots past a token's selected K hold expert -1 and weight 0.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from enum import Enum

import torch

from . import _native as N


class RoutingMode(str, Enum):
    NATURAL = "natural"
    FIXED = "fixed"
    ADAPTIVE = "adaptive"


_MODE_CODE = {RoutingMode.NATURAL: 0, RoutingMode.FIXED: 1, RoutingMode.ADAPTIVE: 2}
K_LADDER = (4, 6, 8, 12, 16)


@dataclass(frozen=True)
class RoutingPolicyConfig:
    """k3x_ref.routing_policy.RoutingPolicyConfig: same fields and defaults."""
    mode: RoutingMode = RoutingMode.NATURAL
    fixed_k: int = 0
    mass_target: float = 0.9
    minimum_boundary_gap: float = 0.0
    quality_floor_k: int = 0

    def to_c(self, collect_diagnostics: bool = False) -> N.RoutingPolicy:
        return N.RoutingPolicy(_MODE_CODE[RoutingMode(self.mode)], int(self.fixed_k),
                               float(self.mass_target), float(self.minimum_boundary_gap),
                               int(self.quality_floor_k), 1 if collect_diagnostics else 0)


@dataclass
class RoutingDecisions:
    """Per-token k3x::RoutingDecision fields for a batch: ``expert_ids`` /
    ``normalized_weights`` are [T, natural_top_k] (natural order, -1 / 0 past
    the selected K), the rest [T]."""
    expert_ids: torch.Tensor
    normalized_weights: torch.Tensor
    selected_k: torch.Tensor
    quality_floor_escalated: torch.Tensor
    normalized_entropy: torch.Tensor
    entropy_effective_support: torch.Tensor
    selected_cumulative_mass: torch.Tensor
    boundary_confidence: torch.Tensor
    natural_top_k: int


def decisions_from(ids: torch.Tensor, weights: torch.Tensor, sel: torch.Tensor,
                   diag: torch.Tensor, natural_top_k: int) -> RoutingDecisions:
    return RoutingDecisions(
        expert_ids=ids, normalized_weights=weights, selected_k=sel[:, 0],
        quality_floor_escalated=sel[:, 1].bool(), normalized_entropy=diag[:, 0],
        entropy_effective_support=diag[:, 1], selected_cumulative_mass=diag[:, 2],
        boundary_confidence=diag[:, 3], natural_top_k=natural_top_k)


def select_routing(scores: torch.Tensor, correction_bias: torch.Tensor, natural_top_k: int,
                   config: RoutingPolicyConfig = RoutingPolicyConfig(),
                   routed_scale: float = 1.0) -> RoutingDecisions:
    """select_routing for every row of ``scores`` [T, E] (sigmoid scores in
    [0, 1], CUDA FP32) with ``correction_bias`` [E]. ``routed_scale`` multiplies
    the weights (1.0 = select_routing's normalized weights). Raises
    Glm5xError(INVALID_STATE) where the reference raises."""
    if scores.ndim != 2 or correction_bias.ndim != 1 or \
            scores.shape[1] != correction_bias.shape[0] or not scores.is_cuda:
        raise ValueError("scores [T, E] and correction_bias [E] on a CUDA device")
    scores = scores.float().contiguous()
    bias = correction_bias.to(scores.device, torch.float32).contiguous()
    T, E = scores.shape
    k = int(natural_top_k)
    dev = scores.device
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    weights = torch.empty((T, k), dtype=torch.float32, device=dev)
    sel = torch.empty((T, 2), dtype=torch.int32, device=dev)
    diag = torch.empty((T, 4), dtype=torch.float32, device=dev)
    pol = config.to_c()
    stream = N.stream_arg(torch.cuda.current_stream(dev).cuda_stream)
    N.check(N.lib().glm5x_select_routing_policy(
        scores.data_ptr(), bias.data_ptr(), T, E, k, ctypes.byref(pol), float(routed_scale),
        ids.data_ptr(), weights.data_ptr(), sel.data_ptr(), diag.data_ptr(), stream))
    return decisions_from(ids, weights, sel, diag, k)
