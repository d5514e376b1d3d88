"""Expert-parallel dispatch / combine (glm5x_moe.ep) on CPU ranks over gloo.

The engine is a CPU stand-in with the same two calls as the GPU engine
(route, forward_expert_rows): every expert is a fixed linear map, so the
expert-parallel result must equal the single-process sum
out[t] = shared(x_t) + sum_s w[t,s] * expert_{ids[t,s]}(x_t) up to the BF16
rounding of the per-destination partial sums on their way back (2^-9
relative each) and FP32 summation order. Covers worlds 2 and 4, ranks that receive no rows, ranks with no local
tokens (both dispatches), tokens whose
experts all live on one rank, uneven token counts per rank, and routes
with empty slots (id -1, as a fixed-K routing policy leaves them), and the
FP4 dispatch (rows quantized by their senders against the slab scales reduced
over the ranks; here with a 4-bit stand-in code and the single-process
result built with the concatenated batch's slab scales), and a forward whose
received rows exceed one rank's capacity, which every rank refuses together
after the same collectives.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, E, K = 32, 16, 4


class FakeEngine:
    def __init__(self, begin: int, count: int, seed: int = 0, keep: int = K) -> None:
        g = torch.Generator().manual_seed(seed)
        self.router = torch.randn(H, E, generator=g)
        self.experts = torch.randn(E, H, H, generator=g) * 0.1
        self.shared = torch.randn(H, H, generator=g) * 0.1
        self.bias = torch.zeros(E)
        self.begin, self.count = begin, count
        self.keep = keep  # slots past `keep` left empty (id -1), as a fixed-K policy does

    def route(self, x: torch.Tensor):
        logits = x.float() @ self.router + self.bias
        # stable: descending score, ties to the lower expert id
        order = torch.sort(-logits, dim=1, stable=True).indices[:, :K]
        w = torch.softmax(torch.gather(logits, 1, order), dim=1)
        if self.keep < K:
            order[:, self.keep:] = -1
            w[:, self.keep:] = 0.0
        return order.to(torch.int32), w

    def forward_expert_rows(self, rows, ids, w, shared_rows=0):
        xf = rows.float()
        out = torch.zeros((rows.shape[0], H))
        for r in range(rows.shape[0]):
            for s in range(K):
                e = int(ids[r, s])
                if e >= 0 and self.begin <= e < self.begin + self.count:
                    out[r] += float(w[r, s]) * (xf[r] @ self.experts[e])
            if r < shared_rows:
                out[r] += xf[r] @ self.shared
        return out

    # FP4 dispatch stand-ins: a 4-bit code per value (two per byte) against
    # the expert's slab amax, so the rows' bytes and sizes travel as NVFP4
    # rows do and the result depends on the reduced slab scale
    def slab_amax(self, x, ids):
        amax = torch.zeros(E)
        xa = x.float().abs().amax(dim=1)
        for t in range(x.shape[0]):
            for s in range(K):
                e = int(ids[t, s])
                if e >= 0:
                    amax[e] = max(float(amax[e]), float(xa[t]))
        return amax

    @staticmethod
    def fake_codes(v, amax):
        return torch.clamp(torch.round(v / max(amax, 1e-30) * 7.0), -7, 7)

    def quantize_rows(self, x, row_token, row_expert, amax):
        n = row_token.numel()
        packed = torch.zeros((n, H // 2), dtype=torch.uint8)
        for r in range(n):
            q = (self.fake_codes(x[int(row_token[r])].float(), float(amax[int(row_expert[r])]))
                 + 8).to(torch.uint8)
            packed[r] = q[0::2] | (q[1::2] << 4)
        return packed, torch.zeros((n, H // 16), dtype=torch.uint8)

    @staticmethod
    def fake_decode(packed_row, amax):
        lo, hi = (packed_row & 15).float() - 8, (packed_row >> 4).float() - 8
        v = torch.stack([lo, hi], dim=1).reshape(-1)
        return v * max(amax, 1e-30) / 7.0

    def forward_quantized_rows(self, x, packed, scales, row_expert, row_weight, amax, group_rows):
        out_local = x.float() @ self.shared
        rows = torch.zeros((packed.shape[0], H))
        for r in range(packed.shape[0]):
            e = int(row_expert[r])
            assert self.begin <= e < self.begin + self.count
            rows[r] = float(row_weight[r]) * (self.fake_decode(packed[r], float(amax[e]))
                                              @ self.experts[e])
        out_groups = torch.zeros((group_rows.shape[0], H))
        for g in range(group_rows.shape[0]):
            for j in range(group_rows.shape[1]):
                if int(group_rows[g, j]) >= 0:
                    out_groups[g] += rows[int(group_rows[g, j])]
        return out_local, out_groups


class CountingEngine(FakeEngine):
    """FakeEngine with the engine's read_ints, counting the reads."""

    reads = 0

    def read_ints(self, t):
        CountingEngine.reads += 1
        return t.reshape(-1).tolist()


def _audit_worker(rank: int, world: int, port: int, fp4: bool, q) -> None:
    """One forward with every other host read-back entry point counted: the
    dispatch must take its split sizes through exactly one read_ints and
    never through tolist / item / nonzero / bincount (each of which reads
    back to the host on a GPU)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from glm5x_moe.ep import ExpertParallelMoE, expert_range
        begin, count = expert_range(rank, world, E)
        eng = CountingEngine(begin, count)
        ep = ExpertParallelMoE(eng, rank=rank, world=world, num_experts=E, top_k=K,
                               hidden_size=H, fp4_dispatch=fp4)
        x = torch.randn(6 + rank, H, generator=torch.Generator().manual_seed(7 + rank))
        x = x.to(torch.bfloat16)
        ids, w = eng.route(x)  # the engine's own calls are not audited
        eng.route = lambda _x, _r=(ids, w): _r
        calls = {"tolist": 0, "item": 0, "nonzero": 0, "bincount": 0}
        saved = (torch.Tensor.tolist, torch.Tensor.item, torch.nonzero, torch.Tensor.nonzero,
                 torch.bincount)

        def wrap(name, fn):
            def f(*a, **kw):
                calls[name] += 1
                return fn(*a, **kw)
            return f

        in_read = [False]
        orig_read = eng.read_ints

        def read(t):
            in_read[0] = True
            try:
                return orig_read(t)
            finally:
                in_read[0] = False
        eng.read_ints = read
        tolist = saved[0]

        def counted_tolist(self_t):
            if not in_read[0]:
                calls["tolist"] += 1
            return tolist(self_t)
        torch.Tensor.tolist = counted_tolist
        torch.Tensor.item = wrap("item", saved[1])
        torch.nonzero = wrap("nonzero", saved[2])
        torch.Tensor.nonzero = wrap("nonzero", saved[3])
        torch.bincount = wrap("bincount", saved[4])
        try:
            CountingEngine.reads = 0
            ep(x)
        finally:
            (torch.Tensor.tolist, torch.Tensor.item, torch.nonzero, torch.Tensor.nonzero,
             torch.bincount) = saved
        q.put((rank, CountingEngine.reads, calls))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, tokens: list[int], skew: bool, q,
            keep: int = K, fp4: bool = False) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from glm5x_moe.ep import ExpertParallelMoE, expert_range
        begin, count = expert_range(rank, world, E)
        eng = FakeEngine(begin, count, keep=keep)
        if skew:
            # every token prefers experts 0..3 (all on rank 0)
            eng.bias[:4] = 50.0
        ep = ExpertParallelMoE(eng, rank=rank, world=world, num_experts=E, top_k=K,
                               hidden_size=H, fp4_dispatch=fp4)
        xs = [torch.randn(tokens[r], H, generator=torch.Generator().manual_seed(100 + r))
              .to(torch.bfloat16) for r in range(world)]
        x = xs[rank]
        out = ep(x)
        ref_eng = FakeEngine(0, E, keep=keep)
        if skew:
            ref_eng.bias[:4] = 50.0
        ids, w = ref_eng.route(x)
        if fp4:
            # one process, the concatenated batch's slab scales
            amax = torch.zeros(E)
            for xr in xs:
                amax = torch.maximum(amax, ref_eng.slab_amax(xr, ref_eng.route(xr)[0]))
            want = x.float() @ ref_eng.shared
            for t in range(x.shape[0]):
                for s in range(K):
                    e = int(ids[t, s])
                    if e >= 0:
                        v = ref_eng.fake_codes(x[t].float(), float(amax[e])) * float(amax[e]) / 7.0
                        want[t] += float(w[t, s]) * (v @ ref_eng.experts[e])
        else:
            want = ref_eng.forward_expert_rows(x, ids, w, shared_rows=x.shape[0])
        if x.shape[0] == 0:  # a rank with no local tokens still serves the others
            assert tuple(out.shape) == (0, H)
            err = 0.0
        else:
            err = float((out - want).abs().max() / want.abs().max())
        q.put((rank, err, ep.last_counts))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,tokens,skew,keep,fp4", [(2, [7, 5], False, K, False),
                                                        (4, [6, 1, 9, 3], False, K, False),
                                                        (2, [8, 4], True, K, False),
                                                        (4, [5, 8, 2, 7], False, 2, False),
                                                        (2, [0, 5], False, K, False),
                                                        (4, [4, 0, 3, 2], False, K, False),
                                                        (2, [7, 5], False, K, True),
                                                        (4, [6, 1, 9, 3], False, 3, True),
                                                        (2, [0, 5], False, K, True),
                                                        (4, [4, 0, 3, 0], False, K, True)])
def test_expert_parallel_matches_single_process(world, tokens, skew, keep, fp4):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, tokens, skew, q, keep, fp4))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, err, counts in res:
        assert err < 5e-3, (rank, err)
    if skew:
        # with all top experts on rank 0, rank 1 receives nothing
        sent, recv = res[1][2]
        assert sum(recv) == 0 and sent[0] == tokens[1]


@pytest.mark.parametrize("T,W,seed", [(1, 2, 0), (37, 4, 1), (64, 8, 2), (5, 4, 3)])
def test_sync_free_pairs_match_plan(T, W, seed):
    """The dispatch pairs built from a known count (prefix sum + scatter)
    equal plan()'s nonzero order: by destination rank, tokens ascending,
    including tokens that reach no rank (all slots empty) and ranks that
    receive nothing."""
    from glm5x_moe.ep import ExpertParallelMoE
    g = torch.Generator().manual_seed(seed)
    ep = ExpertParallelMoE(FakeEngine(0, E), rank=0, world=W, num_experts=E, top_k=K,
                           hidden_size=H)
    ids = torch.randint(0, E // 2, (T, K), generator=g).to(torch.int32)  # upper ranks idle
    ids[::3, 1:] = -1
    if T > 2:
        ids[2, :] = -1
    d_ref, t_ref, c_ref = ep.plan(ids)
    mask = ep._dest_mask(ids)
    assert torch.equal(mask.sum(dim=0), c_ref)
    counts = ep._host_ints(torch.cat([c_ref, c_ref]))
    assert counts[:W] == c_ref.tolist()
    d, t = ep._pairs(mask, sum(counts[:W]))
    assert torch.equal(d, d_ref) and torch.equal(t, t_ref)


@pytest.mark.parametrize("fp4", [False, True])
def test_dispatch_reads_counts_once(fp4):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_audit_worker, args=(r, 2, port, fp4, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for rank, reads, calls in sorted(q.get(timeout=10) for _ in range(2)):
        assert reads == 1, (rank, reads)
        assert all(v == 0 for v in calls.values()), (rank, calls)


def _capacity_worker(rank: int, world: int, port: int, fp4: bool, q) -> None:
    """Rank 1's engine takes at most 10 rows per call; rank 0 has 12 tokens
    with all their experts on rank 1. Every rank must raise the capacity
    error (none may block in a collective the others skipped), and a
    forward within capacity must still work afterwards."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from glm5x_moe.ep import ExpertParallelMoE, expert_range
        begin, count = expert_range(rank, world, E)
        eng = FakeEngine(begin, count)
        eng.bias[E // 2:E // 2 + K] = 50.0  # every token's top-k on rank 1
        ep = ExpertParallelMoE(eng, rank=rank, world=world, num_experts=E, top_k=K,
                               hidden_size=H, fp4_dispatch=fp4,
                               max_rows=1000 if rank == 0 else 10)
        x = torch.randn(12 if rank == 0 else 0, H,
                        generator=torch.Generator().manual_seed(rank)).to(torch.bfloat16)
        raised = ""
        try:
            ep(x)
        except ValueError as e:
            raised = str(e)
        small = torch.randn(2 if rank == 0 else 0, H,
                            generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
        out = ep(small)
        q.put((rank, raised, tuple(out.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fp4", [False, True])
def test_capacity_overflow_raises_on_every_rank(fp4):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_capacity_worker, args=(r, 2, port, fp4, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(2))
    for rank, raised, shape in res:
        assert "EXCEED_MAX_TOKENS" in raised, (rank, raised)
    assert res[0][2] == (2, H) and res[1][2] == (0, H)
