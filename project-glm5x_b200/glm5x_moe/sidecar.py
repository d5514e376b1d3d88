"""Packed expert sidecars (.pn4 / .pm4), the reference's GLM5XPackedExpertCache
file layout (reference/glm5x_ref/packed_cache.py:192-214, 327-404, 407-617),
read by the library's C++ reader (glm5x_sidecar_open): every check of the
reference's get / _decode_role in the same order, CRC32C of every section.

``read_sidecar`` returns the three roles (gate, up, down) as host bytes;
``GLM5XMoELayer.load_sidecar`` admits a file straight into an engine.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

from . import _native as N

_PRECISION = {"nvfp4": N.PRECISION_NVFP4, "mxfp4": N.PRECISION_MXFP4}


@dataclass(frozen=True)
class SidecarRole:
    """One projection of a sidecar: packed E2M1 bytes [rows, cols/2] and its
    scales (NVFP4: blocked E4M3 + FP32 global; MXFP4: row-major E8M0)."""

    precision: str
    shape: tuple[int, int]
    group_size: int
    packed: bytes
    scales: bytes
    global_scale: float


def sidecar_path(root: str | Path, key: tuple[int, int], precision: str) -> Path:
    """root / "layer-LLLL-expert-EEEE.<pn4|pm4>" (GLM5XPackedExpertCache._path)."""
    buf = ctypes.create_string_buffer(4096)
    N.check(N.lib().glm5x_sidecar_path(str(root).encode(), int(key[0]), int(key[1]),
                                       _PRECISION[precision], buf, len(buf)))
    return Path(buf.value.decode())


def read_sidecar(path: str | Path, precision: str | None = None,
                 source_digest: str | None = None) -> list[SidecarRole]:
    """The (gate, up, down) roles of a checked sidecar. Raises Glm5xError
    whose message starts with the reference's error code name (for example
    GLM5X_PACKED_CACHE_PACKED_CRC) where the reference's get() would miss."""
    h = ctypes.c_void_p()
    N.check(N.lib().glm5x_sidecar_open(str(path).encode(),
                                       -1 if precision is None else _PRECISION[precision],
                                       None if source_digest is None else source_digest.encode(),
                                       ctypes.byref(h)))
    try:
        roles = []
        for r in range(3):
            info = N.SidecarRole()
            N.check(N.lib().glm5x_sidecar_get_role(h, r, ctypes.byref(info)))
            roles.append(SidecarRole(
                precision="nvfp4" if info.precision == N.PRECISION_NVFP4 else "mxfp4",
                shape=(int(info.rows), int(info.cols)), group_size=int(info.group_size),
                packed=ctypes.string_at(info.packed, info.packed_bytes),
                scales=ctypes.string_at(info.scales, info.scale_bytes),
                global_scale=float(info.global_scale)))
        return roles
    finally:
        N.lib().glm5x_sidecar_close(h)
