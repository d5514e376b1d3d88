"""The peer-memory expert-parallel layer (glm5x_moe_ep_*,
PeerExpertParallelMoE) on one GPU (world 1: every exchange kernel runs, the
peer being the rank itself), NVFP4 and MXFP4 experts, against the FP32
oracle, over forwards of both buffer parities and a forward without local
tokens; and its argument checks. Bit-equality with the NCCL all-to-all path
(ep.py) is checked in test_gpu_ep.py, with one and with two GPUs.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from moe_fixtures import bf16_to_np, make_expert, make_expert_mxfp4, oracle_forward

pytestmark = pytest.mark.gpu

H, I, E, K = 512, 512, 16, 4


@pytest.mark.parametrize("precision", ["nvfp4", "mxfp4"])
def test_peer_ep_single_rank_matches_oracle(precision):
    from glm5x_moe.ep_peer import PeerExpertParallelMoE
    Tcap = 64
    ep = PeerExpertParallelMoE(rank=0, world=1, max_local_tokens=Tcap, hidden_size=H,
                               intermediate_size=I, num_experts=E, top_k=K, precision=precision)
    make = make_expert if precision == "nvfp4" else make_expert_mxfp4
    fn = O.nvfp4_expert_dequant_oracle if precision == "nvfp4" else O.mxfp4_expert_oracle
    deq = {}
    for e in list(range(E)) + [-1]:
        ex, deq[e] = make(H, I, 8100 + e)
        ep.engine.load_expert(e, ex)
    g = torch.Generator().manual_seed(21)
    router = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.rand(E, generator=g) * 0.2 - 0.1
    ep.engine.set_router(router, bias)
    shared = deq.pop(-1)
    for T in (Tcap, 0, 37, Tcap):
        hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
        out = ep(hidden.cuda())
        ep.check()
        assert tuple(out.shape) == (T, H)
        if T == 0:
            continue
        ids, w = ep.engine.route(hidden.cuda())
        want, _ = oracle_forward(bf16_to_np(hidden), ids.cpu().numpy(), w.cpu().numpy(), deq,
                                 shared, expert_fn=fn)
        max_rel, _, cos = O.relative_error(out.cpu().numpy(), want)
        assert max_rel <= 1e-2 and cos >= 0.9999, (precision, T, max_rel, cos)
    ep.close()


def test_peer_ep_rejects_bad_arguments():
    from glm5x_moe._native import Glm5xError
    from glm5x_moe.ep_peer import PeerExpertParallelMoE
    with pytest.raises(ValueError, match="DIVISIBLE"):
        PeerExpertParallelMoE(rank=0, world=3, max_local_tokens=8, hidden_size=H,
                              intermediate_size=I, num_experts=E, top_k=K)
    ep = PeerExpertParallelMoE(rank=0, world=1, max_local_tokens=8, hidden_size=H,
                               intermediate_size=I, num_experts=E, top_k=K)
    with pytest.raises(Glm5xError, match="max_local_tokens"):
        ep(torch.zeros((9, H), dtype=torch.bfloat16, device="cuda"))
    ep.close()
