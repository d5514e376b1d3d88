"""MXFP4 experts admitted from a .k3x container (glm5x_moe_load_expert_k3x):
the same layer with the same experts loaded from memory gives bit-identical
outputs, and both match the MXFP4 expert oracle (
max rel err <= 1e-2, cosine >= 0.9999)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from k3x_fixture import write_mxfp4_experts
from moe_fixtures import bf16_to_np, make_expert_mxfp4, oracle_forward

pytestmark = pytest.mark.gpu


def test_experts_from_k3x_match_memory_admission(tmp_path):
    from glm5x_moe.k3x import K3xFile
    from glm5x_moe.layer import GLM5XMoELayer
    H, I, E, k, T = 512, 512, 16, 2, 40
    mk = lambda: GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=k,
                               has_shared=True, max_tokens=T, precision="mxfp4")
    direct, from_file = mk(), mk()
    experts, deq, stored = {}, {}, {}
    for e in list(range(E)) + [-1]:
        ex, dq = make_expert_mxfp4(H, I, 600 + e)
        experts[e], deq[e] = ex, dq
        direct.load_expert(e, ex)
        if e < 4:  # experts 0-3 and the shared one go through the container
            prefix = (f"model.layers.0.feed_forward.experts.{e}" if e >= 0
                      else "model.layers.0.feed_forward.shared_experts.0")
            stored[prefix] = (e, {role: (q.packed.cpu().numpy(), q.scales.cpu().numpy(), q.shape)
                                  for role, q in (("gate", ex.gate_proj), ("up", ex.up_proj),
                                                  ("down", ex.down_proj))})
        else:
            from_file.load_expert(e, ex)
    path = tmp_path / "experts.k3x"
    write_mxfp4_experts(path, stored)
    with K3xFile(path, verify=True) as f:
        for prefix, (e, _) in stored.items():
            from_file.load_expert_k3x(e, f, prefix)
    rng = np.random.default_rng(9)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    ids[:, 0] = rng.integers(0, 4, T)  # every token also uses a container expert
    ids[:, 1] = np.where(ids[:, 1] == ids[:, 0], (ids[:, 0] + 5) % E, ids[:, 1])
    w = (rng.random((T, k)) + 0.25).astype(np.float32)
    hidden = torch.randn(T, H, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    a = direct.forward_routed(hidden.cuda(), torch.from_numpy(ids), torch.from_numpy(w))
    b = from_file.forward_routed(hidden.cuda(), torch.from_numpy(ids), torch.from_numpy(w))
    direct.check()
    from_file.check()
    assert torch.equal(a, b)
    shared = deq.pop(-1)
    want, _ = oracle_forward(bf16_to_np(hidden), ids, w, deq, shared,
                             expert_fn=O.mxfp4_expert_oracle)
    max_rel, _, cos = O.relative_error(b.cpu().numpy(), want)
    assert max_rel <= 1e-2 and cos >= 0.9999, (max_rel, cos)
    # a routed-expert prefix that is absent, and an NVFP4 engine, are refused
    from glm5x_moe._native import Glm5xError
    with K3xFile(path, verify=False) as f:
        with pytest.raises(Glm5xError, match="TENSOR_NOT_FOUND"):
            from_file.load_expert_k3x(5, f, "model.layers.0.feed_forward.experts.9")
        nv = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=k,
                           has_shared=False, max_tokens=8)
        with pytest.raises(Glm5xError):
            nv.load_expert_k3x(0, f, "model.layers.0.feed_forward.experts.0")
        nv.close()
    direct.close()
    from_file.close()
