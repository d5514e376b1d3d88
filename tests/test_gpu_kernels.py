"""GPU parity: the stand-alone kernels of libglm5x_moe.so, called through the
C ABI, against the oracle and the reference's golden fixtures. Integer and
byte outputs (packed FP4, scale bytes, routing ids, permutation) must match
bit for bit; decoded values bit for bit as well.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from glm5x_moe import _native as N

pytestmark = pytest.mark.gpu

NV_CASES = ["kat", "seed41", "w_mse", "ragged_mse", "ragged_max", "adv_max", "adv_mse", "act"]
MX_CASES = ["kat_codes", "kat_12", "kat_chunks", "kat_row", "seed31_max", "seed31_mse", "w_max",
            "w_mse", "near_pow2"]


def _s():
    return N.stream_arg(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("name", NV_CASES)
def test_gpu_nvfp4_pack_matches_reference(golden, name):
    from glm5x_moe.nvfp4 import quantize_nvfp4_weight, dequantize_nvfp4
    src = torch.from_numpy(golden[f"nv_{name}_src"]).cuda()
    mode = "mse" if "mse" in name else "max_abs"
    w = quantize_nvfp4_weight(src, scale_mode=mode)
    assert np.array_equal(w.packed.cpu().numpy(), golden[f"nv_{name}_packed"])
    assert np.array_equal(w.scale_bytes().cpu().numpy(), golden[f"nv_{name}_scales"])
    assert np.float32(w.global_scale.item()).view(np.uint32) == \
        golden[f"nv_{name}_global"].view(np.uint32)[0]
    deq = dequantize_nvfp4(w).cpu().numpy()
    assert np.array_equal(deq.view(np.uint32), golden[f"nv_{name}_deq"].view(np.uint32))


@pytest.mark.parametrize("mode", ["max_abs", "mse"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gpu_nvfp4_pack_random_matches_oracle(mode, dtype):
    from glm5x_moe.nvfp4 import quantize_nvfp4_weight
    g = torch.Generator().manual_seed(99)
    for rows, cols, scale in [(256, 6144, 0.02), (384, 2048, 1.0), (130, 96, 30.0)]:
        src = (torch.randn(rows, cols, generator=g) * scale).to(dtype)
        if dtype == torch.float32:
            src[0, :16] = 0
            src[1, :32] *= 1e-6
        w = quantize_nvfp4_weight(src.cuda(), scale_mode=mode)
        p, bl, gl, _ = O.nvfp4_quantize(src.to(torch.float32).numpy(), mode)
        assert np.array_equal(w.packed.cpu().numpy(), p), (rows, cols)
        assert np.array_equal(w.scale_bytes().cpu().numpy(), bl), (rows, cols)
        assert np.float32(w.global_scale.item()) == np.float32(gl)


@pytest.mark.parametrize("name", MX_CASES)
def test_gpu_mxfp4_matches_reference(golden, name):
    from glm5x_moe.nvfp4 import decode_mxfp4, encode_mxfp4
    src = torch.from_numpy(golden[f"mx_{name}_src"]).cuda()
    mode = "mse" if "mse" in name else "max_abs"
    packed, scales = encode_mxfp4(src, 32, scale_mode=mode)
    assert np.array_equal(packed.cpu().numpy(), golden[f"mx_{name}_packed"])
    assert np.array_equal(scales.cpu().numpy(), golden[f"mx_{name}_scales"])
    deq = decode_mxfp4(packed, scales, *src.shape).cpu().numpy()
    assert np.array_equal(deq.view(np.uint32), golden[f"mx_{name}_deq"].view(np.uint32))


def test_gpu_mxfp4_random_and_contract():
    from glm5x_moe.nvfp4 import decode_mxfp4, encode_mxfp4
    g = torch.Generator().manual_seed(5)
    for mode in ("max_abs", "mse"):
        src = torch.randn(64, 2048, generator=g) * 0.02
        p, s = encode_mxfp4(src.cuda(), 32, scale_mode=mode)
        po, so = O.mxfp4_encode(src.numpy(), 32, mode)
        assert np.array_equal(p.cpu().numpy(), po) and np.array_equal(s.cpu().numpy(), so)
    # reserved scale 0xFF is rejected (tests/cuda/test_cuda_mxfp4.cu:21-94)
    with pytest.raises(ValueError, match="0xff"):
        decode_mxfp4(torch.zeros(16, dtype=torch.uint8, device="cuda"),
                     torch.full((1,), 255, dtype=torch.uint8, device="cuda"), 1, 32)
    with pytest.raises(ValueError, match="group_size"):
        decode_mxfp4(torch.zeros(15, dtype=torch.uint8, device="cuda"),
                     torch.zeros(1, dtype=torch.uint8, device="cuda"), 1, 30)
    # columns beyond one block (tests/cuda/test_cuda_mxfp4.cu:96-119)
    packed = torch.zeros(160, dtype=torch.uint8)
    packed[128] = 0x21
    w = decode_mxfp4(packed.cuda(), torch.full((10,), 127, dtype=torch.uint8, device="cuda"),
                     1, 320)
    x = torch.zeros(320)
    x[256], x[257] = 2.0, 3.0
    assert float((w.cpu() @ x)[0]) == 4.0


def test_gpu_select_routing_bit_exact():
    from glm5x_moe import _native as N
    rng = np.random.default_rng(17)
    T, E, k = 700, 256, 8
    scores = rng.random((T, E)).astype(np.float32)
    scores[::3] = np.round(scores[::3] * 16) / 16  # exact ties
    bias = ((rng.random(E) - 0.5) * 0.2).astype(np.float32)
    bias[:64] = 0
    for scale in (1.0, 2.5):
        ids = torch.zeros((T, k), dtype=torch.int32, device="cuda")
        w = torch.zeros((T, k), dtype=torch.float32, device="cuda")
        s_d = torch.from_numpy(scores).cuda()
        b_d = torch.from_numpy(bias).cuda()
        N.check(N.lib().glm5x_select_routing(s_d.data_ptr(), b_d.data_ptr(), T, E, k, scale,
                                             ids.data_ptr(), w.data_ptr(), _s()))
        ids_h, w_h = ids.cpu().numpy(), w.cpu().numpy()
        for t in range(T):
            ro, wo = O.select_routing(scores[t], bias, k)
            assert np.array_equal(ids_h[t], ro), t
            assert np.array_equal(w_h[t], (wo * np.float32(scale)).astype(np.float32)), t


@pytest.mark.parametrize("T,E,k", [(1, 8, 2), (64, 256, 8), (256, 256, 8), (300, 256, 8),
                                   (1000, 64, 4)])
def test_gpu_expert_major_plan(T, E, k):
    from glm5x_moe import _native as N
    rng = np.random.default_rng(T)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    counts, starts, tok, slot, pos = O.expert_major_layout(ids, E, align=128)
    rows = int(starts[-1] + (counts[-1] + 127) // 128 * 128)
    d_ids = torch.from_numpy(ids).cuda()
    cnt = torch.zeros(E, dtype=torch.int32, device="cuda")
    st = torch.zeros(E + 1, dtype=torch.int32, device="cuda")
    ps = torch.zeros((T, k), dtype=torch.int32, device="cuda")
    rt = torch.full((rows + 256,), -1, dtype=torch.int32, device="cuda")
    N.check(N.lib().glm5x_expert_major_plan(d_ids.data_ptr(), T, k, E, cnt.data_ptr(),
                                            st.data_ptr(), ps.data_ptr(), rt.data_ptr(), _s()))
    assert np.array_equal(cnt.cpu().numpy(), counts)
    assert np.array_equal(st.cpu().numpy()[:E], starts)
    assert int(st.cpu().numpy()[E]) == rows
    assert np.array_equal(ps.cpu().numpy(), pos)
    rt_h = rt.cpu().numpy()[:rows]
    valid = tok >= 0
    assert np.array_equal(rt_h[valid], tok[valid])


def _tie_hidden(T, K, rng):
    """BF16 rows whose slab amax is 2688 (global scale exactly 1) and whose
    16-blocks have dyadic maxima, so values divided by their block scale land
    exactly on the E2M1 decision thresholds (0.25, 0.75, ..., 5) where the
    reference's argmin (ties to the lower code) and round-to-nearest-even
    differ, plus signed zeros and saturating values."""
    vals = np.array([0.0, -0.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 0.5, 1.0, 3.0,
                     0.125, 0.7, 1.8, 4.5, 5.5], dtype=np.float32)
    x = rng.choice(vals, size=(T, K // 16, 16)) * rng.choice([-1.0, 1.0], size=(T, K // 16, 16))
    x[:, :, 0] = 6.0  # block max 6 * 2^j below: the E4M3 block scale is 2^j exactly
    x *= (2.0 ** rng.integers(-3, 4, size=(T, K // 16, 1))).astype(np.float32)
    x = x.reshape(T, K)
    x[:, 7] = 2688.0  # every token (so every slab) has amax 2688
    return torch.from_numpy(x.astype(np.float32)).to(torch.bfloat16)


@pytest.mark.parametrize("kind,K,misalign", [("random", 6144, 0), ("ties", 512, 0),
                                             ("ties", 2048, 1)])
def test_gpu_slab_quantize_matches_oracle(kind, K, misalign):
    """Expert-major slab quantization (the activation / intermediate quantizer
    of the forward path) is bit-exact against the oracle, on random data and
    on data built to hit every E2M1 tie; misalign=1 offsets the scale buffer
    by one byte (byte-wise scale stores)."""
    from glm5x_moe import _native as N
    rng = np.random.default_rng(8)
    T, E, k = 96, 16, 4
    if kind == "random":
        hidden = torch.randn(T, K, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16)
        hidden[3] *= 40  # one loud token changes its slabs' global scales
    else:
        hidden = _tie_hidden(T, K, rng)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    counts, starts, tok, slot, pos = O.expert_major_layout(ids, E, align=128)
    rows = int(starts[-1] + (counts[-1] + 127) // 128 * 128)
    hd = hidden.cuda()
    packed = torch.zeros((rows, K // 2), dtype=torch.uint8, device="cuda")
    scales_buf = torch.zeros(O.blocked_size(rows, K // 16) + 16, dtype=torch.uint8, device="cuda")
    scales = scales_buf[misalign:misalign + O.blocked_size(rows, K // 16)]
    gl = torch.zeros(E, dtype=torch.float32, device="cuda")
    rt = torch.from_numpy(np.where(tok >= 0, tok, 0).astype(np.int32)).cuda()
    # keep every device tensor referenced until the call returns
    st_d = torch.from_numpy(np.append(starts, rows).astype(np.int32)).cuda()
    cnt_d = torch.from_numpy(counts.astype(np.int32)).cuda()
    N.check(N.lib().glm5x_nvfp4_quantize_slabs_bf16(
        hd.data_ptr(), K, rt.data_ptr(), st_d.data_ptr(), cnt_d.data_ptr(), E, rows,
        packed.data_ptr(), scales.data_ptr(), gl.data_ptr(), _s()))
    p_h, s_h, g_h = packed.cpu().numpy(), scales.cpu().numpy(), gl.cpu().numpy()
    x = hidden.to(torch.float32).numpy()
    sf_rm = O.from_blocked(s_h, rows, K // 16)
    for e in range(E):
        n = int(counts[e])
        if n == 0:
            continue
        seg = tok[starts[e]:starts[e] + n]
        p, _, g, rm = O.nvfp4_quantize(x[seg], "max_abs")
        assert np.float32(g_h[e]) == np.float32(g), e
        assert np.array_equal(p_h[starts[e]:starts[e] + n], p), e
        assert np.array_equal(sf_rm[starts[e]:starts[e] + n], rm), e
        # N padding rows are zero
        pad = (n + 7) // 8 * 8
        assert not p_h[starts[e] + n:starts[e] + pad].any()
