"""Packed expert sidecars into a real engine (glm5x_moe_load_sidecar): NVFP4
(.pn4) and MXFP4 (.pm4) experts written in the reference's
GLM5XPackedExpertCache layout (tests/sidecar_fixture.py, pinned to files the
reference wrote, tests/test_sidecar.py) must give a layer output bit-identical
to admitting the same matrices from device memory; a corrupted file is
refused with the reference's error and leaves its slot unloaded.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from moe_fixtures import make_expert, make_expert_mxfp4
from sidecar_fixture import mxfp4_role, nvfp4_role, write_sidecar

pytestmark = pytest.mark.gpu

H, I, E, K, T = 512, 512, 16, 2, 40
DIGEST = "glm5x-b200-gpu-sidecar-test"


def _layer(precision):
    from glm5x_moe.layer import GLM5XMoELayer
    return GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=K,
                         has_shared=True, max_tokens=T, precision=precision)


def _b(t: torch.Tensor) -> bytes:
    return t.detach().contiguous().view(torch.uint8).cpu().numpy().tobytes()


def _roles(ex, precision):
    mats = (ex.gate_proj, ex.up_proj, ex.down_proj)
    shapes = ((I, H), (I, H), (H, I))
    if precision == "nvfp4":
        return [nvfp4_role(_b(m.packed), _b(m.scale_bytes()), float(m.global_scale.item()), s)
                for m, s in zip(mats, shapes)]
    return [mxfp4_role(_b(m.packed), _b(m.scales), s) for m, s in zip(mats, shapes)]


@pytest.mark.parametrize("precision", ["nvfp4", "mxfp4"])
def test_sidecar_admission_is_bit_identical(tmp_path, precision):
    from glm5x_moe.sidecar import sidecar_path
    mem, disk = _layer(precision), _layer(precision)
    make = make_expert if precision == "nvfp4" else make_expert_mxfp4
    for e in list(range(E)) + [-1]:
        ex, _ = make(H, I, 600 + e)
        mem.load_expert(e, ex)
        key = (7, e if e >= 0 else E)  # the shared expert under the next free id
        path = sidecar_path(tmp_path, key, precision)
        write_sidecar(path, precision, DIGEST, _roles(ex, precision))
        disk.load_sidecar(e, path)
    g = torch.Generator().manual_seed(12)
    router = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16)
    bias = torch.rand(E, generator=g) * 0.2 - 0.1
    for layer in (mem, disk):
        layer.set_router(router, bias)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    a, b = mem(hidden), disk(hidden)
    assert torch.equal(a.topk_indices, b.topk_indices)
    assert torch.equal(a.output, b.output)
    mem.close()
    disk.close()


def test_corrupted_sidecar_leaves_the_slot_unloaded(tmp_path):
    from glm5x_moe._native import Glm5xError
    from glm5x_moe.sidecar import sidecar_path
    layer = _layer("nvfp4")
    ex, _ = make_expert(H, I, 77)
    path = sidecar_path(tmp_path, (1, 0), "nvfp4")
    write_sidecar(path, "nvfp4", DIGEST, _roles(ex, "nvfp4"))
    data = bytearray(path.read_bytes())
    data[-5] ^= 0x40  # inside the down projection's scales
    path.write_bytes(bytes(data))
    with pytest.raises(Glm5xError) as ei:
        layer.load_sidecar(0, path)
    assert ei.value.code == 11 and "GLM5X_PACKED_CACHE_QPARAM_CRC" in str(ei.value)
    with pytest.raises(Glm5xError, match="FORMAT"):  # an MXFP4 engine refuses a .pn4
        mx = _layer("mxfp4")
        try:
            write_sidecar(path, "nvfp4", DIGEST, _roles(ex, "nvfp4"))
            mx.load_sidecar(0, path)
        finally:
            mx.close()
    ids = torch.zeros((T, K), dtype=torch.int32)
    ids[:, 1] = 1
    with pytest.raises(Glm5xError, match="not loaded"):
        layer.forward_routed(torch.zeros((T, H), dtype=torch.bfloat16, device="cuda"), ids,
                             torch.ones((T, K)))
    layer.close()
