"""NVFP4 / MXFP4 packing on the GPU, mirroring the reference's Python API.

Same names, argument meaning and error strings as
``reference/glm5x_ref/nvfp4.py`` (GLM5XNVFP4Weight, quantize_nvfp4_weight,
dequantize_nvfp4) and ``reference/k3x_ref/mxfp4.py`` (encode_mxfp4,
decode_mxfp4), but every byte is produced by this library's CUDA kernels
through the C ABI. Tensors must live on a CUDA device; there is no CPU path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _native as N

_BLOCK_SIZE = 16


def _ceil_div(value: int, divisor: int) -> int:
    return (value + divisor - 1) // divisor


def _stream() -> ctypes.c_void_p:
    return N.stream_arg(torch.cuda.current_stream().cuda_stream)


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"GLM5X_{what}_CUDA_REQUIRED")


@dataclass(frozen=True)
class GLM5XNVFP4Weight:
    """Packed NVFP4 [out, in] weight with blocked E4M3 scales
    (reference/glm5x_ref/nvfp4.py:58-98)."""

    packed: torch.Tensor
    scales: torch.Tensor
    global_scale: torch.Tensor
    shape: tuple[int, int]

    def __post_init__(self) -> None:
        if self.packed.dtype != torch.uint8 or self.packed.ndim != 2:
            raise ValueError("GLM5X_NVFP4_PACKED_SHAPE")
        if self.scales.dtype not in (torch.float8_e4m3fn, torch.uint8) or self.scales.ndim != 1:
            raise ValueError("GLM5X_NVFP4_SCALE_DTYPE")
        if self.global_scale.dtype != torch.float32 or self.global_scale.numel() != 1:
            raise ValueError("GLM5X_NVFP4_GLOBAL_SCALE")
        rows, cols = (int(self.shape[0]), int(self.shape[1]))
        if cols % _BLOCK_SIZE or cols % 2 or tuple(self.packed.shape) != (rows, cols // 2):
            raise ValueError("GLM5X_NVFP4_WEIGHT_ALIGNMENT")
        expected = _ceil_div(rows, 128) * _ceil_div(cols // _BLOCK_SIZE, 4) * 32 * 16
        if int(self.scales.numel()) != expected:
            raise ValueError("GLM5X_NVFP4_SCALE_SHAPE")

    def num_bytes(self) -> int:
        return int(self.packed.numel()) + int(self.scales.numel()) + 4

    def scale_bytes(self) -> torch.Tensor:
        return self.scales.view(torch.uint8)

    def matrix(self) -> N.Nvfp4Matrix:
        """C-ABI view of this weight (device pointers)."""
        return N.Nvfp4Matrix(self.packed.data_ptr(), self.scale_bytes().data_ptr(),
                             float(self.global_scale.item()), int(self.shape[0]),
                             int(self.shape[1]))


def quantize_nvfp4_weight(weight: torch.Tensor, *, device=None, scale_mode: str = "mse",
                          chunk_rows: int = 128) -> GLM5XNVFP4Weight:
    """Quantize a row-major weight on the GPU and retain its global scale
    (quantize_nvfp4_weight, nvfp4.py:180-198; `chunk_rows` is accepted for
    signature parity and does not change the result)."""
    del chunk_rows
    source = torch.as_tensor(weight)
    if device is not None:
        source = source.to(device=device)
    _require_cuda(source, "NVFP4")
    if source.ndim != 2 or not source.is_floating_point():
        raise ValueError("GLM5X_NVFP4_SOURCE_MATRIX")
    rows, cols = (int(source.shape[0]), int(source.shape[1]))
    if rows <= 0 or cols <= 0 or cols % _BLOCK_SIZE or cols % 2:
        raise ValueError("GLM5X_NVFP4_SOURCE_ALIGNMENT")
    if scale_mode not in {"max_abs", "mse"}:
        raise ValueError("GLM5X_NVFP4_SCALE_MODE")
    mode = N.SCALE_MSE if scale_mode == "mse" else N.SCALE_MAX_ABS
    dev = source.device
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=dev)
    scales = torch.empty(_ceil_div(rows, 128) * _ceil_div(cols // 16, 4) * 512,
                         dtype=torch.uint8, device=dev)
    g = torch.empty((), dtype=torch.float32, device=dev)
    L = N.lib()
    with torch.cuda.device(dev):
        if source.dtype == torch.bfloat16:
            src = source.contiguous()
            st = L.glm5x_nvfp4_quantize_bf16(src.data_ptr(), rows, cols, mode, packed.data_ptr(),
                                             scales.data_ptr(), g.data_ptr(), _stream())
        else:
            src = source.to(torch.float32).contiguous()
            st = L.glm5x_nvfp4_quantize_f32(src.data_ptr(), rows, cols, mode, packed.data_ptr(),
                                            scales.data_ptr(), g.data_ptr(), _stream())
    if st != 0:
        if st == 16:
            raise ValueError("GLM5X_NVFP4_SOURCE_FINITE")
        N.check(st)
    return GLM5XNVFP4Weight(packed=packed, scales=scales.view(torch.float8_e4m3fn),
                            global_scale=g, shape=(rows, cols))


def dequantize_nvfp4(weight: GLM5XNVFP4Weight) -> torch.Tensor:
    """Decode an NVFP4 weight to FP32 on the GPU (nvfp4.py:201-217)."""
    _require_cuda(weight.packed, "NVFP4")
    rows, cols = weight.shape
    out = torch.empty((rows, cols), dtype=torch.float32, device=weight.packed.device)
    with torch.cuda.device(weight.packed.device):
        N.check(N.lib().glm5x_nvfp4_dequantize(
            weight.packed.data_ptr(), weight.scale_bytes().data_ptr(),
            float(weight.global_scale.item()), rows, cols, out.data_ptr(), _stream()))
    return out


def encode_mxfp4(values: torch.Tensor, group_size: int = 32, *, scale_mode: str = "max_abs",
                 chunk_groups: int = 8192) -> tuple[torch.Tensor, torch.Tensor]:
    """E2M1/E8M0 encode on the GPU (k3x_ref/mxfp4.py:31-107); returns device
    tensors (packed uint8 [rows*cols/2], scales uint8 [rows*cols/group])."""
    del chunk_groups
    if values.ndim != 2:
        raise ValueError("values must be a two-dimensional matrix")
    rows, cols = values.shape
    if rows <= 0 or cols <= 0 or group_size <= 0:
        raise ValueError("rows, cols, and group_size must be positive")
    if cols % group_size or cols % 2:
        raise ValueError("cols must align to group_size and nibble pairs")
    if scale_mode not in {"max_abs", "mse"}:
        raise ValueError("scale_mode must be max_abs or mse")
    if not values.is_floating_point():
        raise ValueError("values must use a floating-point dtype")
    _require_cuda(values, "MXFP4")
    src = values.to(torch.float32).contiguous()
    packed = torch.empty(rows * cols // 2, dtype=torch.uint8, device=src.device)
    scales = torch.empty(rows * cols // group_size, dtype=torch.uint8, device=src.device)
    mode = N.SCALE_MSE if scale_mode == "mse" else N.SCALE_MAX_ABS
    with torch.cuda.device(src.device):
        st = N.lib().glm5x_mxfp4_encode_f32(src.data_ptr(), rows, cols, group_size, mode,
                                            packed.data_ptr(), scales.data_ptr(), _stream())
    if st == 15:
        msg = N.lib().glm5x_last_error_message().decode()
        word = int(msg.rsplit("0x", 1)[-1].rstrip(")"), 16) if "0x" in msg else 0
        raise ValueError("values must be finite" if word & 0x2
                         else "values exceed the E8M0 exponent range")
    N.check(st)
    return packed, scales


def decode_mxfp4(packed: torch.Tensor, scales: torch.Tensor, rows: int, cols: int,
                 group_size: int = 32) -> torch.Tensor:
    """E2M1 x 2^(s-127) decode on the GPU (mxfp4.py:110-144); rejects 0xFF."""
    if rows <= 0 or cols <= 0 or group_size <= 0:
        raise ValueError("rows, cols, and group_size must be positive")
    if cols % group_size or cols % 2:
        raise ValueError("cols must align to group_size and nibble pairs")
    if packed.numel() != rows * cols // 2:
        raise ValueError(f"packed length must be {rows * cols // 2}")
    if scales.numel() != rows * cols // group_size:
        raise ValueError(f"scale length must be {rows * cols // group_size}")
    _require_cuda(packed, "MXFP4")
    out = torch.empty((rows, cols), dtype=torch.float32, device=packed.device)
    with torch.cuda.device(packed.device):
        st = N.lib().glm5x_mxfp4_decode(packed.contiguous().data_ptr(),
                                        scales.contiguous().data_ptr(), rows, cols, group_size,
                                        out.data_ptr(), _stream())
    if st == 15:
        raise ValueError("E8M0 scale 0xff is reserved")
    N.check(st)
    return out


@dataclass(frozen=True)
class GLM5XMXFP4Weight:
    """One MXFP4 matrix on the device: packed E2M1 codes [rows * cols / 2]
    (low nibble first) and row-major E8M0 scales [rows * cols / 32], the
    layout of encode_mxfp4 (k3x_ref/mxfp4.py:31-107) and of .pm4 sidecars."""

    packed: torch.Tensor
    scales: torch.Tensor
    shape: tuple[int, int]

    def __post_init__(self) -> None:
        rows, cols = self.shape
        if self.packed.numel() != rows * cols // 2 or self.scales.numel() != rows * cols // 32:
            raise ValueError("GLM5X_MXFP4_WEIGHT_SHAPE")
        if self.packed.dtype != torch.uint8 or self.scales.dtype != torch.uint8:
            raise ValueError("GLM5X_MXFP4_WEIGHT_DTYPE")

    def matrix(self) -> N.Mxfp4Matrix:
        rows, cols = self.shape
        return N.Mxfp4Matrix(self.packed.data_ptr(), self.scales.data_ptr(), rows, cols, 32)


def quantize_mxfp4_weight(weight: torch.Tensor, *, scale_mode: str = "max_abs"
                          ) -> GLM5XMXFP4Weight:
    """Encode a [rows, cols] CUDA matrix to MXFP4 (group 32) on the GPU."""
    packed, scales = encode_mxfp4(weight, 32, scale_mode=scale_mode)
    return GLM5XMXFP4Weight(packed.contiguous(), scales.contiguous(),
                            (int(weight.shape[0]), int(weight.shape[1])))
