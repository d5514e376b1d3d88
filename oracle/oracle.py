"""CPU oracle for the routed-expert MoE path -- TEST INFRASTRUCTURE ONLY.

numpy/ctypes front end over ``oracle/liboracle.so`` (the C restatement in
``glm5x_oracle.c``) and, when present, ``oracle/_ref/libk3x_ref.so`` (the
reference's own C++ CPU sources behind ``ref_shim.cpp``). Only tests/,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import this module,
always as the checker, never as the product path.

Parity pinning: ``tests/test_oracle_golden.py`` checks every function here
against fixtures produced by the reference itself (``tests/golden/``) and
against ``libk3x_ref.so``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = None
_REF = None

E2M1_VALUES = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32,
)

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_VERIFY_ARGS = [ctypes.c_uint32, _u32p, ctypes.c_int, ctypes.c_int, ctypes.c_uint32, _u32p,
                ctypes.c_int, ctypes.POINTER(ctypes.c_int), _u32p]
_POLICY_ARGS = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                ctypes.c_float, ctypes.c_float, ctypes.c_int, _i32p, _f32p, _i32p, _f32p]


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            raise RuntimeError(f"oracle library missing: {path} (run make -f oracle/Makefile)")
        _LIB = ctypes.CDLL(str(path))
        L = _LIB
        L.orc_e4m3_encode.restype = ctypes.c_uint8
        L.orc_e4m3_encode.argtypes = [ctypes.c_float]
        L.orc_e4m3_decode.restype = ctypes.c_float
        L.orc_e4m3_decode.argtypes = [ctypes.c_uint8]
        L.orc_e2m1_encode.restype = ctypes.c_int
        L.orc_e2m1_encode.argtypes = [ctypes.c_float]
        L.orc_nvfp4_quantize.restype = ctypes.c_int
        L.orc_nvfp4_quantize.argtypes = [_f32p, _i64, _i64, ctypes.c_int, _u8p, _u8p,
                                         ctypes.POINTER(ctypes.c_float)]
        L.orc_blocked_size.restype = _i64
        L.orc_blocked_size.argtypes = [_i64, _i64]
        L.orc_to_blocked.restype = None
        L.orc_to_blocked.argtypes = [_u8p, _i64, _i64, _u8p]
        L.orc_from_blocked.restype = None
        L.orc_from_blocked.argtypes = [_u8p, _i64, _i64, _u8p]
        L.orc_nvfp4_dequantize.restype = None
        L.orc_nvfp4_dequantize.argtypes = [_u8p, _u8p, ctypes.c_float, _i64, _i64, _f32p]
        L.orc_mxfp4_encode.restype = ctypes.c_int
        L.orc_mxfp4_encode.argtypes = [_f32p, _i64, _i64, ctypes.c_int, ctypes.c_int, _u8p, _u8p]
        L.orc_mxfp4_decode.restype = ctypes.c_int
        L.orc_mxfp4_decode.argtypes = [_u8p, _u8p, _i64, _i64, ctypes.c_int, _f32p]
        L.orc_select_routing.restype = ctypes.c_int
        L.orc_select_routing.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, _i32p, _f32p]
        L.orc_select_routing_policy.restype = ctypes.c_int
        L.orc_select_routing_policy.argtypes = _POLICY_ARGS
        L.orc_verify_greedy_target_block.restype = ctypes.c_int
        L.orc_verify_greedy_target_block.argtypes = _VERIFY_ARGS
        L.orc_route_tokens.restype = ctypes.c_int
        L.orc_route_tokens.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_float, ctypes.c_void_p, _i32p, _f32p]
        L.orc_dense_silu_mlp.restype = None
        L.orc_dense_silu_mlp.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _f32p]
        L.orc_matmul_nt.restype = None
        L.orc_matmul_nt.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _f32p]
    return _LIB


def ref_lib() -> ctypes.CDLL | None:
    """The reference's compiled CPU path (oracle/_ref), or None if not built."""
    global _REF
    if _REF is None:
        path = HERE / "_ref" / "libk3x_ref.so"
        if not path.exists():
            return None
        _REF = ctypes.CDLL(str(path))
        R = _REF
        R.ref_select_routing.restype = ctypes.c_int
        R.ref_select_routing.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, _i32p, _f32p]
        R.ref_select_routing_policy.restype = ctypes.c_int
        R.ref_select_routing_policy.argtypes = _POLICY_ARGS
        R.ref_verify_greedy_target_block.restype = ctypes.c_int
        R.ref_verify_greedy_target_block.argtypes = _VERIFY_ARGS
        R.ref_k3x_open.restype = ctypes.c_int
        R.ref_k3x_open.argtypes = [ctypes.c_char_p, ctypes.c_int]
        R.ref_k3x_read.restype = ctypes.c_int
        R.ref_k3x_read.argtypes = [ctypes.c_char_p, ctypes.c_uint64, _u8p, ctypes.c_uint64, _u8p,
                                   ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64),
                                   ctypes.POINTER(ctypes.c_uint64)]
        R.ref_decode_mxfp4.restype = ctypes.c_int
        R.ref_decode_mxfp4.argtypes = [_u8p, _u8p, _i64, _i64, _i64, _f32p]
        R.ref_dense_silu_mlp.restype = ctypes.c_int
        R.ref_dense_silu_mlp.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _f32p]
        R.ref_expert_major_plan.restype = ctypes.c_int
        R.ref_expert_major_plan.argtypes = [_i32p, _f32p, ctypes.c_int, ctypes.c_int, _i32p,
                                            _i32p, _i32p, _i32p, _f32p]
    return _REF


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _u8(a) -> np.ndarray:
    if isinstance(a, (bytes, bytearray, memoryview)):
        return np.frombuffer(bytes(a), dtype=np.uint8).copy()
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint8))


# ---------------------------------------------------------------- scalars
def e4m3_encode(x: float) -> int:
    return int(lib().orc_e4m3_encode(float(x)))


def e4m3_decode(code: int) -> float:
    return float(lib().orc_e4m3_decode(int(code)))


def e4m3_decode_array(codes: np.ndarray) -> np.ndarray:
    table = np.array([lib().orc_e4m3_decode(i) for i in range(256)], dtype=np.float32)
    return table[np.asarray(codes, dtype=np.uint8)]


def e2m1_encode(x: float) -> int:
    return int(lib().orc_e2m1_encode(float(x)))


# ---------------------------------------------------------------- NVFP4
def blocked_size(rows: int, cols: int) -> int:
    return int(lib().orc_blocked_size(rows, cols))


def to_blocked(rm: np.ndarray) -> np.ndarray:
    rm = np.ascontiguousarray(rm, dtype=np.uint8)
    rows, cols = rm.shape
    out = np.zeros(blocked_size(rows, cols), dtype=np.uint8)
    lib().orc_to_blocked(rm, rows, cols, out)
    return out


def from_blocked(bl: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.zeros((rows, cols), dtype=np.uint8)
    lib().orc_from_blocked(np.ascontiguousarray(bl, dtype=np.uint8), rows, cols, out)
    return out


def nvfp4_quantize(src, scale_mode: str = "mse"):
    """_quantize_payload + _to_blocked: returns (packed [R, C/2] u8, blocked
    E4M3 scales (1-D u8), global scale float, row-major scales [R, C/16])."""
    x = _f32(src)
    rows, cols = x.shape
    packed = np.zeros((rows, cols // 2), dtype=np.uint8)
    scales = np.zeros((rows, cols // 16), dtype=np.uint8)
    g = ctypes.c_float()
    rc = lib().orc_nvfp4_quantize(x, rows, cols, 1 if scale_mode == "mse" else 0, packed,
                                  scales, ctypes.byref(g))
    if rc:
        raise ValueError(f"orc_nvfp4_quantize failed ({rc})")
    return packed, to_blocked(scales), float(g.value), scales


def nvfp4_dequantize(packed, blocked, g: float, rows: int, cols: int) -> np.ndarray:
    out = np.zeros((rows, cols), dtype=np.float32)
    lib().orc_nvfp4_dequantize(_u8(packed), _u8(blocked), float(g), rows, cols, out)
    return out


# ---------------------------------------------------------------- MXFP4
def mxfp4_encode(src, group: int = 32, scale_mode: str = "max_abs"):
    x = _f32(src)
    rows, cols = x.shape
    packed = np.zeros(rows * cols // 2, dtype=np.uint8)
    scales = np.zeros(rows * cols // group, dtype=np.uint8)
    rc = lib().orc_mxfp4_encode(x, rows, cols, group, 1 if scale_mode == "mse" else 0, packed,
                                scales)
    if rc:
        raise ValueError(f"orc_mxfp4_encode failed ({rc})")
    return packed, scales


def mxfp4_decode(packed, scales, rows: int, cols: int, group: int = 32) -> np.ndarray:
    out = np.zeros((rows, cols), dtype=np.float32)
    rc = lib().orc_mxfp4_decode(_u8(packed), _u8(scales), rows, cols, group, out)
    if rc:
        raise ValueError(f"orc_mxfp4_decode failed ({rc})")
    return out


# ---------------------------------------------------------------- routing
def select_routing(scores, bias, k: int):
    s, b = _f32(scores), _f32(bias)
    ids = np.zeros(k, dtype=np.int32)
    w = np.zeros(k, dtype=np.float32)
    if lib().orc_select_routing(s, b, s.size, k, ids, w):
        raise ValueError("invalid routing")
    return ids, w


ROUTING_MODES = {"natural": 0, "fixed": 1, "adaptive": 2}


def select_routing_policy(scores, bias, k: int, mode: str = "natural", fixed_k: int = 0,
                          mass_target: float = 0.9, minimum_boundary_gap: float = 0.0,
                          quality_floor_k: int = 0, use_reference: bool = False):
    """select_routing with a policy for one token (routing_policy.cpp:31-159):
    (ids [k] with -1 past the selected K, weights [k], selected_k, escalated,
    diag [4] = normalized entropy, effective support, selected mass, boundary
    confidence). `use_reference` runs the reference's own C++ (oracle/_ref)
    instead of the C restatement. Raises ValueError where the reference fails."""
    s, b = _f32(scores), _f32(bias)
    ids = np.zeros(k, dtype=np.int32)
    w = np.zeros(k, dtype=np.float32)
    sel = np.zeros(2, dtype=np.int32)
    diag = np.zeros(4, dtype=np.float32)
    L = ref_lib() if use_reference else lib()
    if L is None:
        raise RuntimeError("oracle/_ref is not built")
    fn = L.ref_select_routing_policy if use_reference else L.orc_select_routing_policy
    if fn(s, b, s.size, k, ROUTING_MODES[mode], fixed_k, float(mass_target),
          float(minimum_boundary_gap), quality_floor_k, ids, w, sel, diag):
        raise ValueError("invalid routing")
    return ids, w, int(sel[0]), bool(sel[1]), diag


def ref_k3x_open(path, verify: bool = True) -> int:
    """k3x::Reader::open of the reference's C++ (oracle/_ref): its ErrorCode."""
    return int(ref_lib().ref_k3x_open(str(path).encode(), 1 if verify else 0))


def ref_k3x_read(path, tensor_id: int, capacity: int = 1 << 24):
    """(status, data bytes, auxiliary bytes) of Reader::read_tensor /
    read_auxiliary in the reference's C++ (oracle/_ref)."""
    data = np.zeros(capacity, dtype=np.uint8)
    aux = np.zeros(capacity, dtype=np.uint8)
    dl, al = ctypes.c_uint64(), ctypes.c_uint64()
    rc = ref_lib().ref_k3x_read(str(path).encode(), tensor_id, data, capacity, aux, capacity,
                                ctypes.byref(dl), ctypes.byref(al))
    return int(rc), data[:dl.value].copy(), aux[:al.value].copy()


def verify_greedy_target_block(anchor: int, candidates, max_draft: int, vocab: int, targets,
                               use_reference: bool = False):
    """(status, accepted, committed tokens) of verify_greedy_target_block;
    `use_reference` runs the reference's own C++ (oracle/_ref)."""
    c = np.ascontiguousarray(np.asarray(candidates, dtype=np.uint32).reshape(-1))
    t = np.ascontiguousarray(np.asarray(targets, dtype=np.uint32).reshape(-1))
    out = np.zeros(c.size + 2, dtype=np.uint32)
    acc = ctypes.c_int(0)
    fn = (ref_lib().ref_verify_greedy_target_block if use_reference
          else lib().orc_verify_greedy_target_block)
    rc = fn(int(anchor), c if c.size else np.zeros(1, np.uint32), c.size, int(max_draft),
            int(vocab), t if t.size else np.zeros(1, np.uint32), t.size, ctypes.byref(acc), out)
    return int(rc), (acc.value if rc == 0 else 0), (out[:acc.value + 1].copy() if rc == 0 else None)


def route_tokens(hidden, router, bias, k: int = 8, routed_scale: float = 2.5,
                 want_logits: bool = False):
    x, w, b = _f32(hidden), _f32(router), _f32(bias)
    T, H = x.shape
    E = w.shape[0]
    ids = np.zeros((T, k), dtype=np.int32)
    wt = np.zeros((T, k), dtype=np.float32)
    logits = np.zeros((T, E), dtype=np.float32) if want_logits else None
    rc = lib().orc_route_tokens(x, w, b, T, H, E, k, float(routed_scale),
                                logits.ctypes.data if logits is not None else None, ids, wt)
    if rc:
        raise ValueError("invalid routing")
    return (ids, wt, logits) if want_logits else (ids, wt)


def expert_major_layout(ids: np.ndarray, num_experts: int, align: int = 128):
    """The device layout this build uses for expert-major token segments:
    experts in ascending id order, each segment's tokens ascending, segment
    starts aligned to `align` rows. Returns (counts [E], starts [E],
    seg_token [rows], seg_slot [rows], pos [T, k]); rows past a segment's
    count are -1. Pure host logic, used to check the device permute."""
    ids = np.asarray(ids)
    T, k = ids.shape
    counts = np.bincount(ids.reshape(-1), minlength=num_experts).astype(np.int64)
    padded = (counts + align - 1) // align * align
    starts = np.concatenate([[0], np.cumsum(padded)[:-1]]).astype(np.int64)
    total = int(padded.sum())
    seg_token = np.full(total, -1, dtype=np.int32)
    seg_slot = np.full(total, -1, dtype=np.int32)
    pos = np.zeros((T, k), dtype=np.int64)
    fill = starts.copy()
    for t in range(T):
        for s in range(k):
            e = int(ids[t, s])
            p = fill[e]
            fill[e] += 1
            seg_token[p] = t
            seg_slot[p] = s
            pos[t, s] = p
    return counts, starts, seg_token, seg_slot, pos


# ---------------------------------------------------------------- dense expert
def dense_silu_mlp(x, gate, up, down) -> np.ndarray:
    x, g, u, d = _f32(x), _f32(gate), _f32(up), _f32(down)
    I, H = g.shape
    out = np.zeros(H, dtype=np.float32)
    lib().orc_dense_silu_mlp(x, g, u, d, H, I, out)
    return out


def matmul_nt(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    M, K = a.shape
    N = b.shape[0]
    out = np.zeros((M, N), dtype=np.float32)
    lib().orc_matmul_nt(a, b, M, N, K, out)
    return out


def bf16_round(x) -> np.ndarray:
    """Round FP32 to the nearest-even BF16 value, returned as FP32."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000))
    return r.astype(np.uint32).view(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    return (x * (np.float32(1.0) / (np.float32(1.0) + np.exp(-x)))).astype(np.float32)


# ---------------------------------------------------------------- MoE layer
def nvfp4_expert_dequant_oracle(slab_bf16: np.ndarray, w13, w2) -> np.ndarray:
    """One routed expert over one token slab, the reference's CUDA NVFP4
    semantics restated in FP32 (layer10_moe.py:711-738 -> nvfp4.py:294-335):
    the slab is quantized once with max_abs and a per-slab global scale, the
    dequantized activation meets the dequantized gate/up weights in an
    FP32-accumulated product (double here), h = silu(gate) * up rounded to
    BF16 (the reference computes it in BF16), h is re-quantized per slab and
    multiplied with the dequantized down weight.

    w13: (gate_deq [I,H], up_deq [I,H]) FP32; w2: down_deq [H,I] FP32.
    Returns [n, H] FP32 expert outputs."""
    gate_deq, up_deq = w13
    n, H = slab_bf16.shape
    p, bl, g, _ = nvfp4_quantize(slab_bf16, "max_abs")
    a = nvfp4_dequantize(p, bl, g, n, H)
    gate = (a.astype(np.float64) @ gate_deq.astype(np.float64).T).astype(np.float32)
    up = (a.astype(np.float64) @ up_deq.astype(np.float64).T).astype(np.float32)
    h = bf16_round(silu(gate) * up)
    I = h.shape[1]
    p2, bl2, g2, _ = nvfp4_quantize(h, "max_abs")
    h_deq = nvfp4_dequantize(p2, bl2, g2, n, I)
    return (h_deq.astype(np.float64) @ w2.astype(np.float64).T).astype(np.float32)


def mxfp4_expert_oracle(x: np.ndarray, w13, w2) -> np.ndarray:
    """One MXFP4 expert over token rows x [n, H] (BF16 values as FP32): the
    reference's MXFP4 expert path restated (layer10_moe.py:571-593 decodes
    the E2M1/E8M0 weights, mxfp4.py:110-144, and runs the expert MLP on the
    decoded weights with unquantized activations, :711-738; the C++ MXFP4
    grid likewise keeps activations in FP32, backend_cuda.cu:1878-2171).
    gate/up/down products accumulate in double, h = silu(gate) * up is rounded
    to BF16 (the reference's linear outputs are BF16).

    w13: (gate_deq [I,H], up_deq [I,H]) FP32; w2: down_deq [H,I] FP32."""
    gate_deq, up_deq = w13
    a = np.asarray(x, dtype=np.float64)
    gate = (a @ gate_deq.astype(np.float64).T).astype(np.float32)
    up = (a @ up_deq.astype(np.float64).T).astype(np.float32)
    h = bf16_round(silu(gate) * up)
    return (h.astype(np.float64) @ w2.astype(np.float64).T).astype(np.float32)


def relative_error(actual: np.ndarray, expected: np.ndarray) -> tuple[float, float, float]:
    """(max |a-e| / max |e|, ||a-e|| / ||e||, cosine similarity)."""
    a = np.asarray(actual, dtype=np.float64).reshape(-1)
    e = np.asarray(expected, dtype=np.float64).reshape(-1)
    denom = max(np.abs(e).max(), 1e-30)
    max_rel = float(np.abs(a - e).max() / denom)
    l2 = float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))
    cos = float(a @ e / max(np.linalg.norm(a) * np.linalg.norm(e), 1e-30))
    return max_rel, l2, cos


if os.environ.get("GLM5X_ORACLE_EAGER"):
    lib()
