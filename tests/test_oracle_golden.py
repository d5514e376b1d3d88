"""CPU tests: the oracle against the reference's own outputs.

Pins every oracle function (oracle/glm5x_oracle.c via oracle/oracle.py) to
fixtures produced by the reference's Python modules
(tests/golden/make_golden.py) and, where built, to the reference's compiled C++
CPU path (oracle/_ref/libk3x_ref.so). Mirrors the reference's known-answer
tests: tests/python/test_ops.py:25-100, tests/cpp/test_ops.cpp:18-22,
tests/cpp/test_routing_policy.cpp:26-46, tests/cpp/test_expert_major.cpp:20-68,
tests/python/test_glm5x_layer10_moe.py:31-78, tests/python/test_glm5x_nvfp4.py:18-27.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O

NV_CASES = ["kat", "seed41", "w_mse", "ragged_mse", "ragged_max", "adv_max", "adv_mse", "act"]
MX_CASES = ["kat_codes", "kat_12", "kat_chunks", "kat_row", "seed31_max", "seed31_mse", "w_max",
            "w_mse", "near_pow2"]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("name", NV_CASES)
def test_nvfp4_pack_matches_reference(golden, name):
    src = golden[f"nv_{name}_src"]
    mode = "mse" if "mse" in name else "max_abs"
    packed, blocked, g, rm = O.nvfp4_quantize(src, mode)
    assert np.array_equal(packed, golden[f"nv_{name}_packed"])
    assert np.array_equal(rm, golden[f"nv_{name}_scales_rm"])
    assert np.array_equal(blocked, golden[f"nv_{name}_scales"])
    assert bits([g])[0] == bits(golden[f"nv_{name}_global"])[0]


@pytest.mark.parametrize("name", NV_CASES)
def test_nvfp4_dequant_matches_reference(golden, name):
    src = golden[f"nv_{name}_src"]
    rows, cols = src.shape
    deq = O.nvfp4_dequantize(golden[f"nv_{name}_packed"], golden[f"nv_{name}_scales"],
                             float(golden[f"nv_{name}_global"][0]), rows, cols)
    assert np.array_equal(bits(deq), bits(golden[f"nv_{name}_deq"]))


def test_nvfp4_kat_row_codes():
    # 0.75 -> 0.5, 1.75 -> 1.5, 3.5 -> 3, 5 -> 4, -0.25 -> +0 (code 0): ties go
    # to the smaller magnitude, not round-to-nearest-even
    row = np.array([[6, 0.75, 0.25, -0.25, 2.5, 5, -0.75, 1.25, 1.75, 3.5, -5, 0, 0, 0, 0, 0]],
                   dtype=np.float32)
    packed, _, g, rm = O.nvfp4_quantize(row, "max_abs")
    codes = np.stack([packed & 15, packed >> 4], axis=-1).reshape(-1)
    assert codes[:12].tolist() == [7, 1, 0, 0, 4, 6, 9, 2, 3, 5, 14, 0]
    assert O.e4m3_decode(int(rm[0, 0])) == 448.0
    assert np.float32(g) == np.float32(0.0022321429569274187)


def test_blocked_layout_round_trip():
    rng = np.random.default_rng(3)
    for rows, cols in [(1, 1), (130, 7), (256, 384), (5, 96)]:
        rm = rng.integers(0, 256, size=(rows, cols), dtype=np.uint8)
        bl = O.to_blocked(rm)
        assert bl.size == O.blocked_size(rows, cols)
        assert np.array_equal(O.from_blocked(bl, rows, cols), rm)


def test_nvfp4_round_trip_error_bound():
    # tests/python/test_glm5x_nvfp4.py:18-27
    rng = np.random.default_rng(41)
    src = O.bf16_round(rng.standard_normal((64, 128)).astype(np.float32))
    p, bl, g, _ = O.nvfp4_quantize(src, "mse")
    deq = O.nvfp4_dequantize(p, bl, g, 64, 128)
    assert np.isfinite(deq).all()
    assert np.linalg.norm(deq - src) / np.linalg.norm(src) < 0.2


def test_e4m3_codec_exhaustive():
    for code in range(256):
        v = O.e4m3_decode(code)
        if np.isnan(v):
            continue
        back = O.e4m3_encode(v)
        assert O.e4m3_decode(back) == v or (v == 0 and back in (0, 0x80))


@pytest.mark.parametrize("name", MX_CASES)
def test_mxfp4_pack_matches_reference(golden, name):
    src = golden[f"mx_{name}_src"]
    mode = "mse" if "mse" in name else "max_abs"
    packed, scales = O.mxfp4_encode(src, 32, mode)
    assert np.array_equal(packed, golden[f"mx_{name}_packed"])
    assert np.array_equal(scales, golden[f"mx_{name}_scales"])
    deq = O.mxfp4_decode(packed, scales, *src.shape)
    assert np.array_equal(bits(deq), bits(golden[f"mx_{name}_deq"]))


def test_mxfp4_literal_kats():
    # tests/python/test_ops.py:25-60 and tests/cpp/test_ops.cpp:18-22
    got = O.mxfp4_decode(bytes([0x10, 0x32] + [0] * 14), bytes([127]), 1, 32)
    assert got[0, :4].tolist() == [0.0, 0.5, 1.0, 1.5]
    got = O.mxfp4_decode(np.full(32, 0x11, np.uint8), np.array([127, 128], np.uint8), 1, 64)
    assert (got[0, :32] == 0.5).all() and (got[0, 32:] == 1.0).all()
    with pytest.raises(ValueError):
        O.mxfp4_decode(np.zeros(16, np.uint8), np.array([255], np.uint8), 1, 32)
    x = np.array([[2.0, 3.0] + [0.0] * 30], np.float32)
    w = O.mxfp4_decode(np.array([0x21] + [0] * 15, np.uint8), np.array([127], np.uint8), 1, 32)
    assert O.matmul_nt(x, w)[0, 0] == 4.0
    _, s = O.mxfp4_encode(np.full((1, 32), 12.0, np.float32))
    assert s.tolist() == [128]


def test_mxfp4_decode_matches_reference_cpp(golden):
    R = O.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built")
    for name in MX_CASES:
        src = golden[f"mx_{name}_src"]
        rows, cols = src.shape
        out = np.zeros((rows, cols), np.float32)
        assert R.ref_decode_mxfp4(golden[f"mx_{name}_packed"], golden[f"mx_{name}_scales"], rows,
                                  cols, 32, out) == 0
        assert np.array_equal(bits(out), bits(golden[f"mx_{name}_deq"]))


def test_select_routing_literal():
    # tests/cpp/test_routing_policy.cpp:30-46
    ids, w = O.select_routing([0.8, 0.8, 0.4, 0.7, 0.2, 0.1], [0, 0, 0.5, 0, 0, 0], 4)
    assert ids.tolist() == [2, 0, 1, 3]
    assert np.allclose(w, np.array([0.4, 0.8, 0.8, 0.7]) / 2.7, atol=1e-6)


def test_select_routing_matches_reference_cpp():
    R = O.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(11)
    for trial in range(300):
        n = 256
        s = rng.random(n).astype(np.float32)
        if trial % 3 == 0:  # plenty of exact ties
            s = (np.round(s * 8) / 8).astype(np.float32)
        b = ((rng.random(n) - 0.5) * 0.2).astype(np.float32)
        if trial % 5 == 0:
            b[:] = 0
        ids_r = np.zeros(8, np.int32)
        w_r = np.zeros(8, np.float32)
        assert R.ref_select_routing(s, b, n, 8, ids_r, w_r) == 0
        ids_o, w_o = O.select_routing(s, b, 8)
        assert np.array_equal(ids_r, ids_o)
        assert np.array_equal(bits(w_r), bits(w_o))


def test_router_matches_reference_python(golden):
    # reference `_route` on seeded GLM-shaped inputs (torch.topk(sorted=False)
    # leaves the slot order unspecified, so sets and per-expert weights)
    hid = (golden["route_hidden_bf16"].astype(np.uint16).astype(np.uint32) << 16).view(np.float32)
    rw = (golden["route_router_bf16"].astype(np.uint16).astype(np.uint32) << 16).view(np.float32)
    ids, w, logits = O.route_tokens(hid, rw, golden["route_bias"], 8, 2.5, want_logits=True)
    assert np.abs(logits - golden["route_logits"]).max() < 1e-4
    for t in range(ids.shape[0]):
        ref = dict(zip(golden["route_indices"][t].tolist(), golden["route_weights"][t].tolist()))
        assert set(ids[t].tolist()) == set(ref)
        for s in range(8):
            assert abs(ref[int(ids[t, s])] - w[t, s]) <= 2e-7


def test_tiny_moe_matches_reference_layer(golden):
    # tests/python/test_glm5x_layer10_moe.py:31-78 through the oracle
    h = golden["moe_tiny_hidden"]
    ids, w = O.route_tokens(h, golden["moe_tiny_router"], golden["moe_tiny_bias"], 2, 2.5)
    assert np.array_equal(np.sort(ids, 1), np.sort(golden["moe_tiny_indices"], 1))
    out = np.zeros_like(h)
    for t in range(h.shape[0]):
        for s in range(2):
            e = int(ids[t, s])
            out[t] += w[t, s] * O.dense_silu_mlp(h[t], golden[f"moe_tiny_gate{e}"],
                                                 golden[f"moe_tiny_up{e}"],
                                                 golden[f"moe_tiny_down{e}"])
        out[t] += O.dense_silu_mlp(h[t], golden["moe_tiny_shared_gate"],
                                   golden["moe_tiny_shared_up"], golden["moe_tiny_shared_down"])
    assert np.allclose(out, golden["moe_tiny_output"], atol=1e-6, rtol=1e-5)


def test_dense_silu_matches_reference_cpp():
    R = O.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(5)
    H, I = 96, 64
    x = rng.standard_normal(H).astype(np.float32)
    g = (rng.standard_normal((I, H)) * 0.1).astype(np.float32)
    u = (rng.standard_normal((I, H)) * 0.1).astype(np.float32)
    d = (rng.standard_normal((H, I)) * 0.1).astype(np.float32)
    ref = np.zeros(H, np.float32)
    assert R.ref_dense_silu_mlp(x, g, u, d, H, I, ref) == 0
    got = O.dense_silu_mlp(x, g, u, d)
    assert np.array_equal(bits(got), bits(ref))


def test_expert_major_plan_reference_cpp():
    # tests/cpp/test_expert_major.cpp:20-68 plus the device layout's ordering
    R = O.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built")
    ids = np.array([[2, 1], [1, 3]], np.int32)
    contrib = np.array([[0.6, 0.4], [0.7, 0.3]], np.float32)
    ge = np.zeros(8, np.int32)
    gs = np.zeros(8, np.int32)
    at = np.zeros(8, np.int32)
    asl = np.zeros(8, np.int32)
    ac = np.zeros(8, np.float32)
    n = R.ref_expert_major_plan(ids, contrib, 2, 2, ge, gs, at, asl, ac)
    assert n == 3 and ge[:3].tolist() == [2, 1, 3] and gs[:3].tolist() == [1, 2, 1]
    assert at[:4].tolist() == [0, 0, 1, 1] and asl[:4].tolist() == [0, 1, 0, 1]
    # the device layout holds the same groups in ascending expert order with
    # the same token order inside each group
    counts, starts, tok, slot, pos = O.expert_major_layout(ids, 4, align=128)
    assert counts.tolist() == [0, 2, 1, 1]
    for g_idx in range(n):
        e = int(ge[g_idx])
        first = int(sum(gs[:g_idx]))
        seg_tok = tok[starts[e]:starts[e] + counts[e]].tolist()
        assert seg_tok == at[first:first + gs[g_idx]].tolist()
