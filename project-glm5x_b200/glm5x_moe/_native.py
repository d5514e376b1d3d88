"""ctypes binding of libglm5x_moe.so (the C ABI declared in include/glm5x_moe.h).

The library is required: importing this module raises if it is missing or
lacks a symbol, so no caller can silently fall back to another code path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

# GLM5X_LIBRARY may point at another build of the same C ABI (e.g. a tuning
# variant); the default is the in-tree build next to this file.
LIB_PATH = Path(os.environ.get("GLM5X_LIBRARY") or
                Path(__file__).resolve().parent / "libglm5x_moe.so")

STATUS_NAMES = {
    0: "OK", 1: "IO_ERROR", 2: "BAD_MAGIC", 3: "UNSUPPORTED_VERSION",
    4: "UNSUPPORTED_REQUIRED_FEATURE", 6: "SUPERBLOCK_CRC_MISMATCH", 7: "TRUNCATED_FILE",
    8: "INVALID_DIRECTORY", 9: "INVALID_EXTENT", 10: "DATA_CRC_MISMATCH",
    11: "AUXILIARY_CRC_MISMATCH", 12: "DIRECTORY_SHA256_MISMATCH", 13: "ROOT_SHA256_MISMATCH",
    14: "TENSOR_NOT_FOUND", 15: "INVALID_MXFP4", 16: "INVALID_STATE",
    17: "BACKEND_UNAVAILABLE", 19: "UNSUPPORTED_ARCHITECTURE", 100: "DEVICE_ERROR",
    101: "OUT_OF_MEMORY", 102: "WAIT_TIMEOUT",
}

NUM_PHASES = 9
PHASE_NAMES = ["row_amax", "router_logits", "topk", "permute", "act_quantize", "gate_up_gemm",
               "h_quantize", "down_gemm", "combine"]

EP_HANDLE_BYTES = 64

PRECISION_NVFP4 = 0
PRECISION_MXFP4 = 1
SCALE_MAX_ABS = 0
SCALE_MSE = 1


class Glm5xError(RuntimeError):
    """A non-OK glm5x_status; `.code` is the numeric status, `.name` its name."""

    def __init__(self, code: int, message: str) -> None:
        self.code = int(code)
        self.name = STATUS_NAMES.get(self.code, f"STATUS_{self.code}")
        super().__init__(f"{self.name}: {message}")


class MoeConfig(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
        ("num_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("has_shared", ctypes.c_int32), ("routed_scaling", ctypes.c_float),
        ("precision", ctypes.c_int32), ("max_tokens", ctypes.c_int32),
        ("expert_begin", ctypes.c_int32), ("expert_count", ctypes.c_int32),
    ]


class Nvfp4Matrix(ctypes.Structure):
    _fields_ = [
        ("packed", ctypes.c_void_p), ("scales", ctypes.c_void_p),
        ("global_scale", ctypes.c_float), ("rows", ctypes.c_int64), ("cols", ctypes.c_int64),
    ]


class Mxfp4Matrix(ctypes.Structure):
    _fields_ = [
        ("packed", ctypes.c_void_p), ("scales", ctypes.c_void_p),
        ("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("group_size", ctypes.c_int64),
    ]


class MoeStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "forward_calls", "kernel_launches", "resident_weight_bytes", "activation_h2d_bytes",
        "device_to_host_bytes", "stream_synchronization_count", "workspace_bytes",
        "loaded_experts")]


class RoutingPolicy(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int32), ("fixed_k", ctypes.c_int32), ("mass_target", ctypes.c_float),
        ("minimum_boundary_gap", ctypes.c_float), ("quality_floor_k", ctypes.c_int32),
        ("collect_diagnostics", ctypes.c_int32),
    ]


class RoutingStats(ctypes.Structure):
    _fields_ = [
        ("decisions", ctypes.c_uint64), ("selected_experts", ctypes.c_uint64),
        ("quality_escalated_decisions", ctypes.c_uint64),
        ("normalized_entropy_sum", ctypes.c_double), ("selected_mass_sum", ctypes.c_double),
        ("boundary_confidence_sum", ctypes.c_double),
    ]


class K3xTensorInfo(ctypes.Structure):
    _fields_ = [
        ("tensor_id", ctypes.c_uint64), ("dtype", ctypes.c_int32),
        ("quantization", ctypes.c_int32), ("rank", ctypes.c_int32), ("layer_id", ctypes.c_int32),
        ("expert_id", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("dimensions", ctypes.c_uint64 * 4), ("data_length", ctypes.c_uint64),
        ("logical_length", ctypes.c_uint64), ("auxiliary_length", ctypes.c_uint64),
    ]


class SidecarRole(ctypes.Structure):
    _fields_ = [
        ("precision", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("group_size", ctypes.c_int64),
        ("packed", ctypes.c_void_p), ("packed_bytes", ctypes.c_int64),
        ("scales", ctypes.c_void_p), ("scale_bytes", ctypes.c_int64),
        ("global_scale", ctypes.c_float),
    ]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F = ctypes.c_float

# name -> argtypes (every function returns glm5x_status unless listed in _RESTYPE)
SIGNATURES = {
    "glm5x_moe_create": [ctypes.POINTER(MoeConfig), ctypes.c_int, ctypes.POINTER(_P)],
    "glm5x_moe_destroy": [_P],
    "glm5x_moe_error_message": [_P],
    "glm5x_last_error_message": [],
    "glm5x_moe_set_router": [_P, _P, _P],
    "glm5x_moe_load_expert_nvfp4": [_P, _I32, ctypes.POINTER(Nvfp4Matrix),
                                    ctypes.POINTER(Nvfp4Matrix), ctypes.POINTER(Nvfp4Matrix)],
    "glm5x_moe_load_expert_nvfp4_device": [_P, _I32, ctypes.POINTER(Nvfp4Matrix),
                                           ctypes.POINTER(Nvfp4Matrix),
                                           ctypes.POINTER(Nvfp4Matrix)],
    "glm5x_moe_load_expert_mxfp4": [_P, _I32, ctypes.POINTER(Mxfp4Matrix),
                                    ctypes.POINTER(Mxfp4Matrix), ctypes.POINTER(Mxfp4Matrix)],
    "glm5x_moe_load_expert_mxfp4_device": [_P, _I32, ctypes.POINTER(Mxfp4Matrix),
                                           ctypes.POINTER(Mxfp4Matrix),
                                           ctypes.POINTER(Mxfp4Matrix)],
    "glm5x_moe_load_sidecar": [_P, _I32, ctypes.c_char_p],
    "glm5x_moe_load_expert_bf16": [_P, _I32, _P, _P, _P, _I32],
    "glm5x_moe_load_expert_bf16_device": [_P, _I32, _P, _P, _P, _I32],
    "glm5x_moe_load_expert_sidecar": [_P, _I32, _P],
    "glm5x_sidecar_open": [ctypes.c_char_p, _I32, ctypes.c_char_p, ctypes.POINTER(_P)],
    "glm5x_sidecar_close": [_P],
    "glm5x_sidecar_get_role": [_P, _I32, ctypes.POINTER(SidecarRole)],
    "glm5x_sidecar_path": [ctypes.c_char_p, _I32, _I32, _I32, ctypes.c_char_p, ctypes.c_size_t],
    "glm5x_k3x_open": [ctypes.c_char_p, _I32, ctypes.POINTER(_P)],
    "glm5x_k3x_close": [_P],
    "glm5x_k3x_tensor": [_P, ctypes.c_char_p, ctypes.POINTER(K3xTensorInfo)],
    "glm5x_k3x_read": [_P, ctypes.c_char_p, _P, ctypes.c_uint64, _P, ctypes.c_uint64],
    "glm5x_moe_load_expert_k3x": [_P, _I32, _P, ctypes.c_char_p],
    "glm5x_moe_forward": [_P, _P, _I64, _P, _P],
    "glm5x_moe_forward_host": [_P, _P, _I64, _P],
    "glm5x_moe_submit_host": [_P, _P, _I64, _P, _P],
    "glm5x_moe_wait_host": [_P, _I64],
    "glm5x_moe_read_ints": [_P, _P, _I64, _P, _P],
    "glm5x_moe_forward_routed": [_P, _P, _I64, _P, _P, _P, _P],
    "glm5x_moe_forward_expert_rows": [_P, _P, _I64, _P, _P, _I64, _P, _P],
    "glm5x_moe_slab_amax": [_P, _P, _I64, _P, _P, _P],
    "glm5x_moe_quantize_rows": [_P, _P, _I64, _P, _P, _I64, _P, _P, _P, _P],
    "glm5x_moe_forward_quantized_rows": [_P, _P, _I64, _P, _P, _P, _P, _I64, _P, _P, _P, _I64,
                                         _I32, _P, _P],
    "glm5x_moe_route": [_P, _P, _I64, _P, _P, _P, _P],
    "glm5x_combine_rows": [_P, _P, _I64, _I32, _I64, _P, _I32, _P],
    "glm5x_verify_greedy_target_blocks": [_P, _P, _P, _P, _I64, _I32, ctypes.c_uint32, _P, _P,
                                          _P, _P],
    "glm5x_moe_last_routing": [_P, _P, _P, _P, _I64],
    "glm5x_moe_ep_create": [ctypes.POINTER(MoeConfig), ctypes.c_int, _I32, _I32, _I64,
                            ctypes.POINTER(_P)],
    "glm5x_moe_ep_handle": [_P, _P],
    "glm5x_moe_ep_connect": [_P, _P],
    "glm5x_moe_create_ep": [ctypes.POINTER(MoeConfig), ctypes.c_int, _P, _I32, _I32, _I64,
                            ctypes.POINTER(_P)],
    "glm5x_moe_ep_engine": [_P],
    "glm5x_moe_ep_forward": [_P, _P, _I64, _P, _P],
    "glm5x_moe_ep_check": [_P],
    "glm5x_moe_ep_error_message": [_P],
    "glm5x_moe_ep_set_profiling": [_P, _I32],
    "glm5x_moe_ep_stage_times": [_P, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(_I32)],
    "glm5x_moe_ep_last_counts": [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I64)],
    "glm5x_moe_ep_destroy": [_P],
    "glm5x_moe_check": [_P],
    "glm5x_moe_get_stats": [_P, ctypes.POINTER(MoeStats)],
    "glm5x_moe_debug_buffer": [_P, _I32, ctypes.POINTER(_P), ctypes.POINTER(ctypes.c_size_t)],
    "glm5x_moe_debug_copy": [_P, _I32, _P, ctypes.c_size_t],
    "glm5x_moe_set_profiling": [_P, _I32],
    "glm5x_moe_phase_times": [_P, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(_I32)],
    "glm5x_moe_get_stream": [_P, ctypes.POINTER(_P)],
    "glm5x_moe_set_tile_n": [_P, _I32],
    "glm5x_moe_set_pair_mma": [_P, _I32],
    "glm5x_moe_set_token_major_down": [_P, _I32],
    "glm5x_moe_set_down_tile_n": [_P, _I32],
    "glm5x_moe_set_weight_tile_rows": [_P, _I32],
    "glm5x_moe_set_pair_wide_stages": [_P, _I32],
    "glm5x_moe_set_pair_tile_order": [_P, _I32, _I32],
    "glm5x_nvfp4_quantize_f32": [_P, _I64, _I64, _I32, _P, _P, _P, _P],
    "glm5x_nvfp4_quantize_bf16": [_P, _I64, _I64, _I32, _P, _P, _P, _P],
    "glm5x_nvfp4_quantize_slabs_bf16": [_P, _I64, _P, _P, _P, _I32, _I64, _P, _P, _P, _P],
    "glm5x_nvfp4_dequantize": [_P, _P, _F, _I64, _I64, _P, _P],
    "glm5x_mxfp4_encode_f32": [_P, _I64, _I64, _I64, _I32, _P, _P, _P],
    "glm5x_mxfp4_decode": [_P, _P, _I64, _I64, _I64, _P, _P],
    "glm5x_select_routing": [_P, _P, _I64, _I32, _I32, _F, _P, _P, _P],
    "glm5x_select_routing_policy": [_P, _P, _I64, _I32, _I32, ctypes.POINTER(RoutingPolicy), _F,
                                    _P, _P, _P, _P, _P],
    "glm5x_moe_set_routing_policy": [_P, ctypes.POINTER(RoutingPolicy)],
    "glm5x_read_bf16_activation": [ctypes.c_char_p, ctypes.c_uint32, ctypes.c_uint32,
                                   ctypes.POINTER(ctypes.c_uint32),
                                   ctypes.POINTER(ctypes.c_uint32), _P, ctypes.c_uint64],
    "glm5x_write_bf16_activation": [ctypes.c_char_p, _P, ctypes.c_uint32, ctypes.c_uint32],
    "glm5x_moe_routing_stats": [_P, ctypes.POINTER(RoutingStats)],
    "glm5x_moe_routing_decisions": [_P, _I64, _P, _P],
    "glm5x_expert_major_plan": [_P, _I64, _I32, _I32, _P, _P, _P, _P, _P],
    "glm5x_expert_major_plan_noalloc": [_P, _I64, _I32, _I32, _P, _P, _P, _P, _P],
}
_RESTYPE = {
    "glm5x_moe_destroy": None,
    "glm5x_k3x_close": None,
    "glm5x_sidecar_close": None,
    "glm5x_moe_ep_destroy": None,
    "glm5x_moe_ep_engine": ctypes.c_void_p,
    "glm5x_moe_ep_error_message": ctypes.c_char_p,
    "glm5x_moe_error_message": ctypes.c_char_p,
    "glm5x_last_error_message": ctypes.c_char_p,
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libglm5x_moe.so once; raise if it is absent or incomplete."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m glm5x_moe.build` "
                "(there is no fallback implementation)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)  # AttributeError if the symbol is missing
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, ctypes.c_int)
        _lib = handle
    return _lib


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy


def stream_arg(handle: int) -> ctypes.c_void_p:
    """A torch stream handle as the C ABI's `stream`: torch's default stream
    has handle 0, which the C ABI would read as "the engine's own stream", so
    it is passed as cudaStreamLegacy instead."""
    return ctypes.c_void_p(handle if handle else CUDA_STREAM_LEGACY)


def check(status: int, engine=None) -> None:
    if status != 0:
        L = lib()
        msg = (L.glm5x_moe_error_message(engine) if engine else L.glm5x_last_error_message())
        raise Glm5xError(status, (msg or b"").decode(errors="replace"))
