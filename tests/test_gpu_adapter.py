"""The k3x::ComputeBackend adapter (project-glm5x_b200/adapter), driven the
way the reference runtime drives its CUDA backend: a plan from the
reference's own build_expert_major_packed_plan (runtime/src/expert_major.cpp)
and a call through k3x::ComputeBackend& to
raw_bf16_situ_mlp_expert_major_with_shared (runtime/include/k3x/backend.hpp:
228-236) with SiLU, BF16 expert views (RawBf16MlpView) and a shared expert.

The adapter packs the views to NVFP4 on first use (the reference's NVFP4
packing) and runs them on libglm5x_moe.so, so its output must equal, bit for
bit, the engine's own forward over the same BF16 experts, stay the same on
a second call (weights resident, cache hits counted), and match the FP32
dequant-matmul oracle within the north-star tolerance.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle as O
from moe_fixtures import bf16_to_np, oracle_forward

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
CHECK = REPO / "oracle" / "_ref" / "libk3x_adapter_check.so"
H, I, E, K, T = 512, 512, 8, 2, 24


def test_compute_backend_adapter_expert_major_with_shared():
    from glm5x_moe import _native as N
    from glm5x_moe.layer import GLM5XMoELayer
    from glm5x_moe.nvfp4 import quantize_nvfp4_weight
    N.lib()
    if not CHECK.exists():
        pytest.fail(f"{CHECK} was not built (needs the reference headers at build time)")
    lib = ctypes.CDLL(str(CHECK))
    g = torch.Generator().manual_seed(91)
    experts = [[(torch.randn(s, generator=g) * 0.02).to(torch.bfloat16)
                for s in ((I, H), (I, H), (H, I))] for _ in range(E + 1)]
    flat = torch.cat([torch.cat([m.reshape(-1) for m in ex]) for ex in experts[:E]])
    shared = torch.cat([m.reshape(-1) for m in experts[E]])
    rng = np.random.default_rng(4)
    ids = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.uint32)
    w = (rng.random((T, K)) + 0.2).astype(np.float32)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
    x = bf16_to_np(hidden)
    out = np.zeros((2, T, H), dtype=np.float32)
    hits = ctypes.c_ulonglong()
    msg = ctypes.create_string_buffer(512)
    rc = lib.adapter_expert_major(
        0, H, I, E, K, T, x.ctypes.data_as(ctypes.c_void_p), ids.ctypes.data_as(ctypes.c_void_p),
        w.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(flat.data_ptr()),
        ctypes.c_void_p(shared.data_ptr()), 2, out.ctypes.data_as(ctypes.c_void_p),
        ctypes.byref(hits), msg, len(msg))
    assert rc == 0, (rc, msg.value)
    assert np.array_equal(out[0], out[1]) and hits.value >= E + 1
    # the engine itself over the same experts (expert e in slot e)
    layer = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=K,
                          has_shared=True, max_tokens=T)
    deq = {}
    for e in range(E + 1):
        slot = e if e < E else -1
        layer.load_expert_bf16(slot, *experts[e])
        q = [quantize_nvfp4_weight(m.cuda(), scale_mode="mse") for m in experts[e]]
        deq[slot] = tuple(O.nvfp4_dequantize(m.packed.cpu().numpy(), m.scale_bytes().cpu().numpy(),
                                             float(m.global_scale.item()), *t.shape)
                          for m, t in zip(q, experts[e]))
    mine = layer.forward_routed(hidden.cuda(), torch.from_numpy(ids.astype(np.int32)),
                                torch.from_numpy(w)).cpu().numpy()
    layer.close()
    assert np.array_equal(out[0], mine)
    sh = deq.pop(-1)
    want, _ = oracle_forward(x, ids.astype(np.int32), w, deq, sh)
    max_rel, _, cos = O.relative_error(out[0], want)
    assert max_rel <= 1e-2 and cos >= 0.9999, (max_rel, cos)
