"""GLM5XACT BF16 activation batch files through the C ABI.

The reference hands hidden states between its Python layer and its C++
runtime in these files: ``write_bf16_activation``
(converter/glm5x_converter/activation.py:21-57) writes the MoE input and the
expected output (reference/glm5x_ref/activation_export.py:99-123), and the
runtime's ``load_glm5x_bf16_activation`` (runtime/src/glm5x_activation.cpp:
53-109) reads them for its GLM expert bench (--input-bf16 / --expected-bf16,
runtime/src/cuda_glm5x_real_expert_bench.cpp:426-458). Same names, same
checks, same error statuses (raised as Glm5xError).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

from . import _native as N


def load_bf16_activation(path: str | Path, expected_token_count: int = 0,
                         expected_hidden_size: int = 0) -> torch.Tensor:
    """Read and verify one batch: BF16 [tokens, hidden] on the CPU."""
    L = N.lib()
    p = str(path).encode()
    t, h = ctypes.c_uint32(), ctypes.c_uint32()
    N.check(L.glm5x_read_bf16_activation(p, expected_token_count, expected_hidden_size,
                                         ctypes.byref(t), ctypes.byref(h), None, 0))
    out = torch.empty((t.value, h.value), dtype=torch.bfloat16)
    N.check(L.glm5x_read_bf16_activation(p, expected_token_count, expected_hidden_size,
                                         ctypes.byref(t), ctypes.byref(h), out.data_ptr(),
                                         out.numel()))
    return out


def write_bf16_activation(path: str | Path, tensor: torch.Tensor) -> None:
    """Write one contiguous [tokens, hidden] BF16 batch (converted to BF16)."""
    work = torch.as_tensor(tensor).detach().to(device="cpu", dtype=torch.bfloat16)
    if work.ndim != 2:
        raise ValueError("activation tensor must be rank-2 [tokens, hidden]")
    work = work.contiguous()
    if work.shape[0] == 0 or work.shape[1] == 0:
        raise ValueError("activation tensor dimensions must be non-zero")
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    N.check(N.lib().glm5x_write_bf16_activation(str(path).encode(), work.data_ptr(),
                                                work.shape[0], work.shape[1]))
