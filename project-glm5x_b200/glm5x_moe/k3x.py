"""K3X v1 checkpoint containers (.k3x) through the C ABI.

The reference runtime keeps model weights in .k3x files (reader:
runtime/src/reader.cpp, k3x::Reader; writer: converter/k3x_converter/
writer.py) with MXFP4 expert projections as UINT8 records (packed E2M1)
carrying an E8M0 auxiliary extent. ``K3xFile`` opens one with the reader's
checks and status codes (raised as Glm5xError), reads records by name, and
``GLM5XMoELayer.load_expert_k3x`` admits an expert's three MXFP4 records.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import _native as N


def fnv1a64(name: str) -> int:
    """Tensor id of a name (converter/k3x_converter/format.py:49-54)."""
    h = 0xCBF29CE484222325
    for byte in name.encode("utf-8"):
        h ^= byte
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


class K3xFile:
    """An open .k3x container; ``verify`` = the reader's checksums mode (every
    extent's CRC32C, directory and root SHA-256), else metadata only."""

    def __init__(self, path: str | Path, verify: bool = True) -> None:
        self._h = ctypes.c_void_p()
        N.check(N.lib().glm5x_k3x_open(str(path).encode(), 1 if verify else 0,
                                       ctypes.byref(self._h)))

    def close(self) -> None:
        if self._h:
            N.lib().glm5x_k3x_close(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self) -> "K3xFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def tensor(self, name: str) -> dict:
        """The tensor record of ``name`` as a dict (dtype 1 FP32, 2 UINT8,
        3 BF16; quantization 1 = MXFP4; ``shape`` = dimensions[:rank])."""
        info = N.K3xTensorInfo()
        N.check(N.lib().glm5x_k3x_tensor(self._h, name.encode(), ctypes.byref(info)))
        out = {f: getattr(info, f) for f, _ in N.K3xTensorInfo._fields_ if f != "dimensions"}
        out["shape"] = tuple(info.dimensions[i] for i in range(info.rank))
        return out

    def read(self, name: str) -> tuple[np.ndarray, np.ndarray | None]:
        """(data bytes, auxiliary bytes or None) of tensor ``name``."""
        rec = self.tensor(name)
        data = np.empty(rec["data_length"], dtype=np.uint8)
        aux = (np.empty(rec["auxiliary_length"], dtype=np.uint8)
               if rec["auxiliary_length"] else None)
        N.check(N.lib().glm5x_k3x_read(self._h, name.encode(), data.ctypes.data, data.size,
                                       aux.ctypes.data if aux is not None else None,
                                       aux.size if aux is not None else 0))
        return data, aux
