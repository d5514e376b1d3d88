"""Generate golden fixtures by running the reference's own Python modules.

Run in a container where the reference project is readable (it is not on the
GPU box; the fixtures it writes are committed next to this script):

    python tests/golden/make_golden.py /path/to/reference

The reference's package `__init__` imports ``google_crc32c``; the pure-Python
stand-in under ``tests/golden/_shims`` is put on ``sys.path`` for that.
Every fixture is seeded and small (KB to a few MB).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    ref = Path(ref_root)
    sys.path[:0] = [str(HERE / "_shims"), str(ref / "reference"), str(ref / "converter")]
    import torch
    import torch.nn.functional as F
    from glm5x_ref.nvfp4 import (_quantize_payload, _to_blocked, dequantize_nvfp4,
                                 quantize_nvfp4_weight)
    from k3x_ref.mxfp4 import decode_mxfp4, encode_mxfp4
    from glm5x_ref.layer10_moe import GLM5XExpertWeights, GLM5XLayer10MoEReference

    torch.set_num_threads(8)
    out: dict[str, np.ndarray] = {}

    # ------------------------------------------------------------- NVFP4
    def nv(name: str, src: torch.Tensor, mode: str) -> None:
        src32 = src.to(torch.float32)
        w = quantize_nvfp4_weight(src32, device="cpu", scale_mode=mode)
        packed, raw, g = _quantize_payload(src32, scale_mode=mode)
        assert torch.equal(_to_blocked(raw).view(torch.uint8), w.scales.view(torch.uint8))
        out[f"nv_{name}_src"] = src32.numpy()
        out[f"nv_{name}_packed"] = w.packed.numpy()
        out[f"nv_{name}_scales"] = w.scales.view(torch.uint8).numpy()
        out[f"nv_{name}_scales_rm"] = raw.view(torch.uint8).numpy()
        out[f"nv_{name}_global"] = np.array([float(w.global_scale)], dtype=np.float32)
        out[f"nv_{name}_deq"] = dequantize_nvfp4(w).numpy()

    kat = torch.tensor([[6, 0.75, 0.25, -0.25, 2.5, 5, -0.75, 1.25, 1.75, 3.5, -5, 0,
                         0, 0, 0, 0]], dtype=torch.float32)
    nv("kat", kat, "max_abs")
    torch.manual_seed(41)
    nv("seed41", torch.randn(64, 128, dtype=torch.bfloat16), "max_abs")
    g = torch.Generator().manual_seed(7)
    nv("w_mse", (torch.randn(128, 256, generator=g) * 0.02).to(torch.bfloat16), "mse")
    nv("ragged_mse", (torch.randn(130, 64, generator=g) * 0.02).to(torch.bfloat16), "mse")
    nv("ragged_max", torch.randn(200, 48, generator=g).to(torch.bfloat16), "max_abs")
    # adversarial: zero blocks, exact E2M1 midpoints, tiny magnitudes, one huge block
    adv = torch.zeros(8, 64)
    adv[1, :16] = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 2)
    adv[1, 16:32] = -adv[1, :16]
    adv[2, :] = 1e-9
    adv[3, :] = torch.linspace(-3, 3, 64)
    adv[4, 5] = 1000.0
    adv[5, :] = torch.randn(64, generator=g) * 1e-4
    adv[6, ::2] = 448.0 * 6
    adv[7, :] = -0.0
    nv("adv_max", adv, "max_abs")
    nv("adv_mse", adv, "mse")
    nv("act", torch.randn(5, 6144, generator=g).to(torch.bfloat16), "max_abs")

    # ------------------------------------------------------------- MXFP4
    def mx(name: str, src: torch.Tensor, mode: str, chunk_groups: int = 8192) -> None:
        src32 = src.to(torch.float32)
        packed, scales = encode_mxfp4(src32, group_size=32, chunk_groups=chunk_groups,
                                      scale_mode=mode)
        out[f"mx_{name}_src"] = src32.numpy()
        out[f"mx_{name}_packed"] = np.frombuffer(packed, dtype=np.uint8).copy()
        out[f"mx_{name}_scales"] = np.frombuffer(scales, dtype=np.uint8).copy()
        rows, cols = src32.shape
        out[f"mx_{name}_deq"] = decode_mxfp4(packed, scales, rows, cols, 32).numpy()

    mx("kat_codes", torch.tensor([[0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0] + [0.0] * 24]),
       "max_abs")
    mx("kat_12", torch.full((1, 32), 12.0), "max_abs")
    mx("kat_chunks", torch.cat((torch.full((1, 32), 1.0), torch.full((1, 32), 2.0))),
       "max_abs", chunk_groups=1)
    mx("kat_row", torch.cat((kat, torch.zeros(1, 16)), dim=1), "max_abs")
    g2 = torch.Generator().manual_seed(31)
    mx("seed31_max", torch.randn((2, 32), generator=g2), "max_abs")
    mx("seed31_mse", torch.randn((2, 32), generator=torch.Generator().manual_seed(31)), "mse")
    mx("w_max", (torch.randn(64, 256, generator=g2) * 0.02).to(torch.bfloat16), "max_abs")
    mx("w_mse", (torch.randn(32, 256, generator=g2) * 0.02).to(torch.bfloat16), "mse")
    # group maxima within a few ulps of 6 * 2^k (the ceil(log2) boundary)
    near = []
    for k in range(-20, 21, 3):
        base = np.float32(6.0 * 2.0 ** k)
        for step in range(-3, 4):
            v = base
            for _ in range(abs(step)):
                v = np.nextafter(v, np.float32(np.inf if step > 0 else 0), dtype=np.float32)
            row = np.linspace(-0.5, 0.5, 32, dtype=np.float32) * base
            row[7] = v
            near.append(row)
    mx("near_pow2", torch.tensor(np.stack(near)), "max_abs")

    # ------------------------------------------------------------- routing
    hidden = torch.tensor([[0.5, -1.0, 0.25], [1.0, 0.25, -0.75]], dtype=torch.float32)
    router = torch.tensor([[1.0, 0.0, 0.0], [0.0, 1.0, 0.0], [0.0, 0.0, 1.0], [-1.0, 0.5, 0.25]],
                          dtype=torch.float32)
    bias = torch.tensor([0.0, 0.1, -0.2, 0.05], dtype=torch.float32)

    def weights(expert_id: int) -> GLM5XExpertWeights:
        base = float(expert_id + 1)
        gate = torch.tensor([[base, 0.5, -0.25], [-0.5, base * 0.25, 0.75]])
        up = torch.tensor([[0.25, base, 0.5], [0.75, -0.5, base * 0.2]])
        down = torch.tensor([[base, -0.25], [0.5, base * 0.1], [0.25, 0.75]])
        return GLM5XExpertWeights(gate_proj=gate, up_proj=up, down_proj=down)

    shared = GLM5XExpertWeights(
        gate_proj=torch.tensor([[0.5, 0.25, -0.5], [0.75, -0.25, 0.5]]),
        up_proj=torch.tensor([[1.0, -0.5, 0.25], [0.25, 0.5, 1.0]]),
        down_proj=torch.tensor([[0.5, -0.25], [0.75, 0.5], [-0.5, 0.25]]))
    model = GLM5XLayer10MoEReference(router_weight=router, correction_bias=bias,
                                     expert_loader=weights, shared_expert=shared, top_k=2)
    res = model(hidden)
    out["moe_tiny_hidden"] = hidden.numpy()
    out["moe_tiny_router"] = router.numpy()
    out["moe_tiny_bias"] = bias.numpy()
    out["moe_tiny_indices"] = res.topk_indices.numpy().astype(np.int32)
    out["moe_tiny_weights"] = res.topk_weights.numpy()
    out["moe_tiny_output"] = res.output.numpy()
    for e in range(4):
        w = weights(e)
        out[f"moe_tiny_gate{e}"] = w.gate_proj.numpy()
        out[f"moe_tiny_up{e}"] = w.up_proj.numpy()
        out[f"moe_tiny_down{e}"] = w.down_proj.numpy()
    out["moe_tiny_shared_gate"] = shared.gate_proj.numpy()
    out["moe_tiny_shared_up"] = shared.up_proj.numpy()
    out["moe_tiny_shared_down"] = shared.down_proj.numpy()

    # GLM-shaped router on seeded synthetic inputs (reference `_route`)
    gr = torch.Generator().manual_seed(2024)
    T, H, E = 48, 6144, 256
    hid = torch.randn(T, H, generator=gr).to(torch.bfloat16)
    rw = (torch.randn(E, H, generator=gr) * 0.02).to(torch.bfloat16)
    rb = (torch.rand(E, generator=gr) * 0.2 - 0.1).to(torch.float32)
    big = GLM5XLayer10MoEReference(router_weight=rw, correction_bias=rb,
                                   expert_loader=weights, shared_expert=shared)
    logits, idx, wts = big._route(hid)
    out["route_hidden_bf16"] = hid.view(torch.int16).numpy()
    out["route_router_bf16"] = rw.view(torch.int16).numpy()
    out["route_bias"] = rb.numpy()
    out["route_logits"] = logits.numpy()
    out["route_indices"] = idx.numpy().astype(np.int32)
    out["route_weights"] = wts.numpy()

    np.savez_compressed(HERE / "reference_golden.npz", **out)
    print("wrote", HERE / "reference_golden.npz", len(out), "arrays")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GLM5X_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: %s <reference project root> (or set GLM5X_REFERENCE_ROOT)" % sys.argv[0])
    main(root)
