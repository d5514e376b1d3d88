"""Host-buffer entry points on the GPU.

glm5x_moe_forward_host follows the reference ComputeBackend convention (host
spans in, an owned host vector out, synchronous per call;
runtime/include/k3x/backend.hpp:220-252). glm5x_moe_submit_host /
glm5x_moe_wait_host pipeline the same work over two staging slots and three
streams. Both must give exactly the device-buffer forward's output, and that
output meets the FP32 dequant-matmul oracle's tolerance.
"""
from __future__ import annotations

import pytest
import torch

import oracle as O
from moe_fixtures import bf16_to_np, make_expert, oracle_forward

pytestmark = pytest.mark.gpu

H, I, E, K = 512, 512, 16, 4
MAX_T = 64


def _layer():
    from glm5x_moe.layer import GLM5XMoELayer
    layer = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=K,
                          has_shared=True, max_tokens=MAX_T)
    deq = {}
    for e in list(range(E)) + [-1]:
        ex, dq = make_expert(H, I, 700 + e)
        layer.load_expert(e, ex)
        deq[e] = dq
    g = torch.Generator().manual_seed(77)
    layer.set_router((torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16),
                     torch.rand(E, generator=g) * 0.2 - 0.1)
    return layer, deq


def _hidden(T, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, H, generator=g).to(torch.bfloat16)


def test_forward_host_equals_device_forward():
    layer, deq = _layer()
    hidden = _hidden(48, 5)
    res = layer(hidden.cuda())
    out = torch.empty((48, H), dtype=torch.float32).pin_memory()
    layer.forward_host(hidden.pin_memory(), out)
    assert torch.equal(out, res.output.cpu())
    shared = deq.pop(-1)
    want, _ = oracle_forward(bf16_to_np(hidden), res.topk_indices.numpy(),
                             res.topk_weights.numpy(), deq, shared)
    max_rel, _, cos = O.relative_error(out.numpy(), want)
    assert max_rel <= 1e-2 and cos >= 0.9999, (max_rel, cos)
    layer.close()


def test_pipelined_host_forward_matches_synchronous():
    """Batches of different sizes in flight together (each staging slot used
    several times, waits lagging two tickets behind), one pair of pageable
    buffers among them: every output equals the synchronous call's."""
    layer, _ = _layer()
    sizes = [48, 17, 64, 1, 33, 64, 5, 40]
    inputs = [_hidden(T, 100 + i) for i, T in enumerate(sizes)]
    want = []
    for x in inputs:
        o = torch.empty((x.shape[0], H), dtype=torch.float32).pin_memory()
        layer.forward_host(x.pin_memory(), o)
        want.append(o.clone())
    pageable = 4
    outs, tickets = [], []
    for i, x in enumerate(inputs):
        if i == pageable:
            xin, o = x.clone(), torch.full((x.shape[0], H), float("nan"))
        else:
            xin = x.pin_memory()
            o = torch.full((x.shape[0], H), float("nan")).pin_memory()
        outs.append(o)
        tickets.append(layer.submit_host(xin, o))
        if i >= 2:
            layer.wait_host(tickets[i - 2])
    for t in tickets[-2:]:
        layer.wait_host(t)
    assert tickets == list(range(len(sizes)))
    for i, (o, w) in enumerate(zip(outs, want)):
        assert torch.equal(o, w), i
    layer.check()
    layer.close()


def test_pipelined_host_forward_errors():
    """Host-side checks of the pipelined API: waits on tickets that were not
    issued, batches over max_tokens, and the ticket sequence after a refused
    submission."""
    from glm5x_moe._native import Glm5xError
    layer, _ = _layer()
    x = _hidden(8, 3).pin_memory()
    o = torch.empty((8, H), dtype=torch.float32).pin_memory()
    with pytest.raises(Glm5xError) as ei:
        layer.wait_host(0)  # nothing submitted yet
    assert ei.value.code == 16  # GLM5X_INVALID_STATE
    big = torch.zeros((MAX_T + 1, H), dtype=torch.bfloat16)
    with pytest.raises(Glm5xError) as ei:
        layer.submit_host(big, torch.empty((MAX_T + 1, H), dtype=torch.float32))
    assert ei.value.code == 9  # GLM5X_INVALID_EXTENT
    t = layer.submit_host(x, o)
    assert t == 0  # the refused batch took no ticket
    layer.wait_host(t)
    with pytest.raises(Glm5xError) as ei:
        layer.wait_host(t + 1)
    assert ei.value.code == 16
    layer.wait_host(t)  # waiting twice is allowed
    want = torch.empty_like(o).pin_memory()
    layer.forward_host(x, want)
    assert torch.equal(o, want)
    layer.close()


def test_read_ints_through_mapped_memory():
    """glm5x_moe_read_ints: device int64 words on the host after the current
    stream's work, written by device stores into mapped page-locked memory."""
    from glm5x_moe._native import Glm5xError
    layer, _ = _layer()
    vals = torch.arange(-5, 3000, 7, dtype=torch.int64, device="cuda") * 1_000_003
    assert layer.read_ints(vals) == vals.cpu().tolist()
    # the read follows work queued before it on the stream
    x = torch.zeros(4096, dtype=torch.int64, device="cuda")
    x += torch.arange(4096, device="cuda")
    assert layer.read_ints(x) == list(range(4096))
    assert layer.read_ints(torch.empty(0, dtype=torch.int64, device="cuda")) == []
    with pytest.raises(Glm5xError) as ei:
        layer.read_ints(torch.zeros(4097, dtype=torch.int64, device="cuda"))
    assert ei.value.code == 9
    layer.close()
