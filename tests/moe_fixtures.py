"""Shared helpers for the GPU parity tests: seeded NVFP4 experts packed by the
library's GPU packer, their oracle dequantization, and the oracle forward of
the routed-expert sublayer (the FP32 dequant-matmul construction of the
reference's tests/python/test_glm5x_nvfp4.py:30-47 applied per expert slab,
layer10_moe.py:791-847 + 954-961)."""
from __future__ import annotations

import numpy as np
import torch

import oracle as O


def bf16_to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).cpu().numpy()


def make_expert(H: int, I: int, seed: int, device="cuda"):
    """Returns (NVFP4Expert on device, (gate_deq, up_deq, down_deq) FP32 host)."""
    from glm5x_moe.layer import NVFP4Expert
    from glm5x_moe.nvfp4 import quantize_nvfp4_weight
    g = torch.Generator(device="cpu").manual_seed(seed)
    mats = []
    deq = []
    for shape in ((I, H), (I, H), (H, I)):
        w = (torch.randn(shape, generator=g) * 0.02).to(torch.bfloat16).to(device)
        q = quantize_nvfp4_weight(w, scale_mode="mse")
        mats.append(q)
        deq.append(O.nvfp4_dequantize(q.packed.cpu().numpy(), q.scale_bytes().cpu().numpy(),
                                      float(q.global_scale.item()), *shape))
    return NVFP4Expert(*mats), tuple(deq)


def make_expert_mxfp4(H: int, I: int, seed: int, device="cuda"):
    """Returns (MXFP4Expert on device, (gate_deq, up_deq, down_deq) FP32 host),
    encoded by the library's GPU MXFP4 encoder (max_abs, group 32) and
    decoded by the oracle."""
    from glm5x_moe.layer import MXFP4Expert
    from glm5x_moe.nvfp4 import quantize_mxfp4_weight
    g = torch.Generator(device="cpu").manual_seed(seed)
    mats, deq = [], []
    for shape in ((I, H), (I, H), (H, I)):
        w = (torch.randn(shape, generator=g) * 0.02).to(torch.bfloat16).to(device)
        q = quantize_mxfp4_weight(w)
        mats.append(q)
        deq.append(O.mxfp4_decode(q.packed.cpu().numpy(), q.scales.cpu().numpy(), *shape))
    return MXFP4Expert(*mats), tuple(deq)


def oracle_forward(hidden: np.ndarray, ids: np.ndarray, weights: np.ndarray,
                   experts_deq: dict, shared_deq=None, expert_fn=None) -> tuple[np.ndarray, dict]:
    """hidden [T, H] (BF16 values as FP32); ids/weights [T, k] (id -1 = an
    empty slot, as a fixed / adaptive routing policy leaves). Returns the
    layer output [T, H] and the per-(token, slot) expert outputs. expert_fn
    defaults to the NVFP4 per-slab oracle."""
    expert_fn = expert_fn or O.nvfp4_expert_dequant_oracle
    T, H = hidden.shape
    out = np.zeros((T, H), dtype=np.float64)
    per = {}
    for e in sorted(set(int(v) for v in ids.reshape(-1) if v >= 0)):  # -1 = empty slot
        tok, slot = np.nonzero(ids == e)
        order = np.argsort(tok, kind="stable")
        tok, slot = tok[order], slot[order]
        gd, ud, dd = experts_deq[e]
        y = expert_fn(hidden[tok], (gd, ud), dd)
        for i, (t, s) in enumerate(zip(tok, slot)):
            per[(int(t), int(s))] = y[i]
            out[t] += np.float64(weights[t, s]) * y[i]
    if shared_deq is not None:
        gd, ud, dd = shared_deq
        out += expert_fn(hidden, (gd, ud), dd)
    return out.astype(np.float32), per
