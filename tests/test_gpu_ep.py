"""Expert-parallel engines on the GPU.

test_expert_rows_single_gpu: one engine holding experts [4, 8) of 8 runs
dispatched rows whose slots name experts held elsewhere (skipped) or -1, and
the shared expert only on the leading rows; checked against the oracle.

test_expert_parallel_two_gpus: two ranks (one process per GPU, NCCL) each
hold half the experts, exchange tokens with glm5x_moe.ep, and must match the
oracle of the same layer (routed-expert slabs across ranks, shared-expert
slab per rank) within the north-star tolerance (needs 2 GPUs); the FP4
dispatch and the peer-memory layer (glm5x_moe_ep_*, PeerExpertParallelMoE:
rows stored into and partial sums pulled from the peers' memory by the
library's kernels) must give the same bits as the BF16 all-to-all dispatch,
over several forwards (both buffer parities) and with a rank that has no
local tokens (one GPU: the same with a single rank).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

import oracle as O
from moe_fixtures import bf16_to_np, make_expert, oracle_forward

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MIN_COS = 0.9999


def _assert_close(got, want, what):
    max_rel, l2, cos = O.relative_error(got, want)
    assert max_rel <= MAX_REL and cos >= MIN_COS, (what, max_rel, l2, cos)


@pytest.mark.parametrize("shared_rows", [30, 0])
def test_expert_rows_single_gpu(shared_rows):
    """shared_rows = 0: only received rows, as on a rank without local tokens."""
    from glm5x_moe.layer import GLM5XMoELayer
    H, I, E, k, R = 512, 512, 8, 2, 70
    layer = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=k,
                          has_shared=True, max_tokens=R, expert_begin=4, expert_count=4)
    deq = {}
    for e in list(range(4, 8)) + [-1]:
        ex, dq = make_expert(H, I, 4000 + e)
        layer.load_expert(e, ex)
        deq[e] = dq
    rng = np.random.default_rng(5)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(R)]).astype(np.int32)
    ids[::7, 1] = -1
    w = rng.random((R, k)).astype(np.float32) + 0.25
    rows = torch.randn(R, H, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    out = layer.forward_expert_rows(rows.cuda(), torch.from_numpy(ids), torch.from_numpy(w),
                                    shared_rows=shared_rows).cpu().numpy()
    layer.check()
    # oracle: held experts only (others contribute zero), shared on rows < 30
    local = np.where((ids >= 4) & (ids < 8), ids, -1)
    x = bf16_to_np(rows)
    want = np.zeros((R, H), np.float32)
    shared = deq.pop(-1)
    for e in range(4, 8):
        tok, slot = np.nonzero(local == e)
        if tok.size:
            y = O.nvfp4_expert_dequant_oracle(x[tok], deq[e][:2], deq[e][2])
            for i, (t, s) in enumerate(zip(tok, slot)):
                want[t] += w[t, s] * y[i]
    if shared_rows:
        want[:shared_rows] += O.nvfp4_expert_dequant_oracle(x[:shared_rows], shared[:2],
                                                            shared[2])
    _assert_close(out, want, "expert rows")
    layer.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_worker(rank, world, port, q):
    import torch.distributed as dist
    from glm5x_moe.ep import ExpertParallelMoE, expert_range
    from glm5x_moe.layer import GLM5XMoELayer
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        H, I, E, k = 512, 512, 16, 4
        tokens = [48 + 16 * r for r in range(world)]
        T = tokens[rank]
        begin, count = expert_range(rank, world, E)
        # room for the local tokens plus every received row: BF16 dispatch
        # sends a token once per rank, FP4 dispatch once per (token, expert)
        ep_layer = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=k,
                                 has_shared=True, max_tokens=T + k * sum(tokens), device=rank,
                                 expert_begin=begin, expert_count=count)
        full = GLM5XMoELayer(hidden_size=H, intermediate_size=I, num_experts=E, top_k=k,
                             has_shared=True, max_tokens=sum(tokens), device=rank)
        deq = {}
        for e in list(range(E)) + [-1]:
            ex, deq[e] = make_expert(H, I, 5000 + e, device=f"cuda:{rank}")
            full.load_expert(e, ex)
            if e < 0 or begin <= e < begin + count:
                ep_layer.load_expert(e, ex)
        g = torch.Generator().manual_seed(11)
        router = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
        bias = torch.rand(E, generator=g) * 0.2 - 0.1
        full.set_router(router, bias)
        ep_layer.set_router(router, bias)
        xs = [torch.randn(tokens[r], H, generator=torch.Generator().manual_seed(100 + r))
              .to(torch.bfloat16) for r in range(world)]
        x = xs[rank].cuda(rank)
        ep = ExpertParallelMoE(ep_layer, rank=rank, world=world, num_experts=E, top_k=k,
                               hidden_size=H)
        got = ep(x).cpu().numpy()
        torch.cuda.synchronize(rank)
        ep_layer.check()
        counts = ep.last_counts
        # FP4 dispatch: the same slabs, so the same bits
        ep4 = ExpertParallelMoE(ep_layer, rank=rank, world=world, num_experts=E, top_k=k,
                                hidden_size=H, fp4_dispatch=True)
        got4 = ep4(x).cpu().numpy()
        torch.cuda.synchronize(rank)
        ep_layer.check()
        fp4_equal = bool(np.array_equal(got, got4))
        # the peer-memory layer: same experts, same router, same bits, on
        # three forwards (parities 1, 0, 1), the middle one with rank 0 empty
        from glm5x_moe.ep_peer import PeerExpertParallelMoE
        peer = PeerExpertParallelMoE(rank=rank, world=world, max_local_tokens=max(tokens),
                                     hidden_size=H, intermediate_size=I, num_experts=E,
                                     top_k=k, device=rank)
        for e in list(range(begin, begin + count)) + [-1]:
            ex, _ = make_expert(H, I, 5000 + e, device=f"cuda:{rank}")
            peer.engine.load_expert(e, ex)
        peer.engine.set_router(router, bias)
        x_b = x[:0] if rank == 0 else x
        want_b = ep(x_b).cpu().numpy()
        peer_equal = []
        for xi, ref in ((x, got), (x_b, want_b), (x, got)):
            out_p = peer(xi).cpu().numpy()
            peer.check()
            peer_equal.append(bool(np.array_equal(out_p, ref)))
        dist.barrier()
        peer.close()
        # Oracle with the parallel layer's slabs: a routed expert's slab holds
        # every rank's tokens routed to it (the same slab as one GPU running
        # the concatenated batch); the shared expert's slab is the rank's own
        # tokens. Routing comes from the single-GPU layer on the concatenated
        # batch (per-token logits do not depend on the other tokens).
        res = full(torch.cat(xs).cuda(rank))
        x_all = bf16_to_np(torch.cat(xs))
        ids = res.topk_indices.numpy()
        w = res.topk_weights.numpy()
        shared = deq.pop(-1)
        routed, _ = oracle_forward(x_all, ids, w, deq, None)
        off = sum(tokens[:rank])
        want = routed[off:off + T] + O.nvfp4_expert_dequant_oracle(bf16_to_np(xs[rank]),
                                                                   shared[:2], shared[2])
        max_rel, l2, cos = O.relative_error(got, want)
        q.put((rank, max_rel, cos, counts, fp4_equal, ep4.last_counts, peer_equal))
        full.close()
        ep_layer.close()
    finally:
        dist.destroy_process_group()


def _run_ep(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for _ in range(world):
        rank, max_rel, cos, counts, fp4_equal, counts4, peer_equal = q.get(timeout=10)
        assert max_rel <= MAX_REL and cos >= MIN_COS, (rank, max_rel, cos, counts)
        assert sum(counts[1]) > 0 and sum(counts4[1]) > 0, (counts, counts4)
        assert fp4_equal, rank
        assert all(peer_equal), (rank, peer_equal)


def test_expert_parallel_fp4_dispatch_one_gpu():
    """The expert-parallel module with one rank: BF16 and FP4 dispatch give
    the same bits, and both match the oracle."""
    _run_ep(1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_two_gpus():
    _run_ep(2)
