"""GPU test of glm5x_expert_major_plan_noalloc, the expert-major plan whose
scratch lives in a fixed __device__ array instead of cudaMalloc'd memory (for
callers whose device memory is owned by another allocator, or that cannot
take cudaFree's device-wide synchronization).

It must give the same plan as glm5x_expert_major_plan on every call,
including back-to-back calls that reuse the shared scratch array; plans are
integer outputs, so the comparison is exact. This file sorts last so a
stop-at-first-failure run has already run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _plan(fn_name, ids, E):
    from glm5x_moe import _native as N
    T, k = ids.shape
    d_ids = torch.from_numpy(ids).cuda()
    cnt = torch.full((E,), -7, dtype=torch.int32, device="cuda")
    st = torch.full((E + 1,), -7, dtype=torch.int32, device="cuda")
    pos = torch.full((T, k), -7, dtype=torch.int32, device="cuda")
    rows = T * k + E * 128 + 256
    rt = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    stream = N.stream_arg(torch.cuda.current_stream().cuda_stream)
    N.check(getattr(N.lib(), fn_name)(d_ids.data_ptr(), T, k, E, cnt.data_ptr(), st.data_ptr(),
                                      pos.data_ptr(), rt.data_ptr(), stream))
    total = int(st[E].item())
    return cnt.cpu().numpy(), st.cpu().numpy(), pos.cpu().numpy(), rt[:total].cpu().numpy()


def test_noalloc_plan_matches_allocating_plan_twice():
    rng = np.random.default_rng(2718)
    cases = [(1000, 256, 8), (77, 64, 4)]  # two calls in a row, different shapes
    for T, E, k in cases:
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
        want = _plan("glm5x_expert_major_plan", ids, E)
        got = _plan("glm5x_expert_major_plan_noalloc", ids, E)
        for w, g in zip(want, got):
            assert np.array_equal(w, g)


def test_noalloc_plan_at_its_limits_then_smaller():
    """The advertised maxima (8192 tokens, 65536 (token, slot) pairs: the
    whole chunk-count, rank and row-weight regions of the scratch array),
    then a smaller multi-chunk plan that must not read the larger call's
    leftover chunk counts."""
    rng = np.random.default_rng(31)
    cases = [(8192, 256, 8), (300, 256, 8)]
    for T, E, k in cases:
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
        want = _plan("glm5x_expert_major_plan", ids, E)
        got = _plan("glm5x_expert_major_plan_noalloc", ids, E)
        for w, g in zip(want, got):
            assert np.array_equal(w, g)


def test_noalloc_plan_rejects_oversize():
    from glm5x_moe import _native as N
    ids = torch.zeros((9000, 8), dtype=torch.int32, device="cuda")
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    st = N.lib().glm5x_expert_major_plan_noalloc(ids.data_ptr(), 9000, 8, 256, dummy.data_ptr(),
                                                 dummy.data_ptr(), dummy.data_ptr(),
                                                 dummy.data_ptr(), None)
    assert st == 9
    assert b"fixed scratch" in N.lib().glm5x_last_error_message()
