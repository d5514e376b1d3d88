"""CPU tests: the C-ABI library loads, exports every declared entry point,
and rejects bad arguments before touching a device (the sidecar reader has
its own tests in test_sidecar.py). No GPU compute is called here.
"""
from __future__ import annotations

import ctypes
import json
import re
import struct
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "glm5x_moe.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(glm5x_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_symbols()
    for required in ["glm5x_moe_create", "glm5x_moe_forward", "glm5x_moe_load_expert_nvfp4",
                     "glm5x_moe_load_sidecar", "glm5x_moe_set_router", "glm5x_moe_last_routing",
                     "glm5x_nvfp4_quantize_f32", "glm5x_mxfp4_decode"]:
        assert required in names


def test_library_exports_every_declared_symbol():
    from glm5x_moe import _native as N
    lib = N.lib()
    handle = ctypes.CDLL(str(N.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(handle, name), name
        assert name in N.SIGNATURES, f"{name} has no ctypes signature"
    assert lib is not None


def test_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from glm5x_moe import _native as N
    cfg = N.MoeConfig(6144, 2048, 256, 8, 1, 2.5, 0, 64, 0, 256)
    h = ctypes.c_void_p()
    st = N.lib().glm5x_moe_create(ctypes.byref(cfg), 0, ctypes.byref(h))
    assert st == 17  # BACKEND_UNAVAILABLE
    assert not h.value


def test_argument_validation_precedes_device_work():
    from glm5x_moe import _native as N
    L = N.lib()
    cfg = N.MoeConfig(6000, 2048, 256, 8, 1, 2.5, 0, 64, 0, 256)  # hidden not /512
    h = ctypes.c_void_p()
    assert L.glm5x_moe_create(ctypes.byref(cfg), 0, ctypes.byref(h)) == 9
    assert b"multiples of 512" in L.glm5x_last_error_message()
    cfg = N.MoeConfig(6144, 2048, 256, 0, 1, 2.5, 0, 64, 0, 256)  # top_k 0
    assert L.glm5x_moe_create(ctypes.byref(cfg), 0, ctypes.byref(h)) == 9
    assert L.glm5x_mxfp4_decode(None, None, 1, 30, 32, None, None) == 15
    assert L.glm5x_select_routing(None, None, 1, 256, 8, 1.0, None, None, None) == 16
