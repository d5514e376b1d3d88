"""Expert parallelism: the MoE sublayer with its routed experts sharded
across ranks (one process per GPU), tokens exchanged by all-to-all.

The reference runs every expert in one process (layer10_moe.py:791-847 +
954-961); this module is the multi-GPU form of the same computation. Rank r
of W holds experts [r * E/W, (r + 1) * E/W) plus a replica of the shared
expert and the full router. A forward on rank r:

1. routes its local tokens (all E experts);
2. dispatch: every (token, destination rank) pair whose token has at least
   one expert on that rank sends the token's BF16 row once, with its top-k
   global ids masked to that rank's experts (-1 elsewhere) and its weights;
   counts go first (all-to-all of int64), then the rows and the id/weight
   words (all-to-all-v);
3. runs its experts over [local tokens; received rows] in one engine call:
   the local tokens take only the shared expert, the received rows only the
   held routed experts;
4. combine: each received row's weighted sum returns to its source
   (all-to-all-v of BF16 rows), where the partial sums of a token are added
   in FP32, in destination-rank order, onto its shared-expert output.

With fp4_dispatch, step 2 sends NVFP4 rows instead: every rank computes the
per-expert max |x| of its tokens (slab_amax) and the ranks reduce it with MAX,
which gives each routed expert's slab scale exactly as one GPU computes it
for the concatenated batch; every (token, expert) pair then travels as that
expert's NVFP4 row (H/2 code bytes + H/16 scale bytes + 12 bytes of expert
id, weight and token instead of 2H bytes per (token, rank)), the receiver
runs its experts on the rows as they are (forward_quantized_rows) and sums
each source token's rows before the return. The result is bit-identical to
the BF16 dispatch.

Every rank takes the same collectives in the same order in every forward,
including ranks without local tokens (both dispatches) and forwards that fail:
the received-row count is checked against the engine's capacity
(`max_rows`, the engine's max_tokens) on every rank, the verdict is reduced
with MAX over the ranks together with the counts, and all ranks raise
together before any row is exchanged.

Everything runs on the caller's current stream; torch.distributed (NCCL on
GPUs) moves the bytes. The engine is any object with route(hidden) ->
(ids, weights) and forward_expert_rows(rows, ids, weights, shared_rows), plus
slab_amax, quantize_rows and forward_quantized_rows for fp4_dispatch.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class ExpertParallelMoE:
    """Dispatch / expert / combine around one rank's engine."""

    def __init__(self, engine, *, rank: int, world: int, num_experts: int, top_k: int,
                 hidden_size: int, group=None, fp4_dispatch: bool = False,
                 max_rows: int | None = None) -> None:
        if num_experts % world:
            raise ValueError("GLM5X_EP_EXPERTS_NOT_DIVISIBLE")
        self.engine = engine
        self.num_experts = num_experts
        # local tokens + received rows one engine call takes (the engine's
        # max_tokens); None = unbounded (host stand-in engines)
        self.max_rows = max_rows if max_rows is not None else getattr(engine, "max_tokens", None)
        self.rank = rank
        self.world = world
        self.per = num_experts // world
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.group = group
        self.fp4_dispatch = fp4_dispatch
        self.last_counts: tuple[list[int], list[int]] | None = None
        self.last_local_assignments = 0
        self._timing = False
        self._stage_ms = [0.0, 0.0, 0.0, 0.0]
        self._pending: list = []
        self._timed = 0

    STAGES = ("route", "dispatch", "experts", "combine")

    def set_timing(self, enable: bool) -> None:
        """Record CUDA events on the current stream at the stage boundaries."""
        self._timing = enable

    def stage_times(self) -> tuple[dict, int]:
        """(milliseconds per stage summed since the last call, forwards)."""
        for evs in self._pending:
            evs[-1].synchronize()
            for i in range(4):
                self._stage_ms[i] += evs[i].elapsed_time(evs[i + 1])
            self._timed += 1
        self._pending = []
        out = (dict(zip(self.STAGES, self._stage_ms)), self._timed)
        self._stage_ms = [0.0, 0.0, 0.0, 0.0]
        self._timed = 0
        return out

    def _mark(self, evs) -> None:
        if evs is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            evs.append(e)

    def plan(self, ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(dest [n], token [n], counts [W]) of the dispatch pairs, ordered by
        destination rank, tokens ascending within a destination. Slots with id
        -1 (left empty by a fixed / adaptive routing policy) go nowhere."""
        T = ids.shape[0]
        valid = ids >= 0
        dest = torch.where(valid, ids.long() // self.per, 0)
        hits = torch.zeros((T, self.world), dtype=torch.int32, device=ids.device)
        hits.scatter_add_(1, dest, valid.to(torch.int32))
        mask = hits > 0
        d_idx, t_idx = mask.t().nonzero(as_tuple=True)
        return d_idx, t_idx, mask.sum(dim=0)

    def _dest_mask(self, ids: torch.Tensor) -> torch.Tensor:
        """[T, W] bool: token t has at least one expert on rank d."""
        valid = ids >= 0
        dest = torch.where(valid, ids.long() // self.per, 0)
        hits = torch.zeros((ids.shape[0], self.world), dtype=torch.int32, device=ids.device)
        hits.scatter_add_(1, dest, valid.to(torch.int32))
        return hits > 0

    @staticmethod
    def _pairs(mask: torch.Tensor, n_pairs: int) -> tuple[torch.Tensor, torch.Tensor]:
        """The (dest, token) pairs of plan() for a known pair count, found by a
        prefix sum and a scatter instead of nonzero (which reads its size back
        to the host)."""
        T = mask.shape[0]
        flat = mask.t().reshape(-1)
        pos = torch.cumsum(flat, 0) - 1
        pos = torch.where(flat, pos, torch.full_like(pos, n_pairs))  # unused slot
        lin = torch.empty(n_pairs + 1, dtype=torch.int64, device=mask.device)
        lin.scatter_(0, pos, torch.arange(flat.numel(), device=mask.device))
        lin = lin[:n_pairs]
        return lin // T, lin % T

    def _host_ints(self, t: torch.Tensor) -> list[int]:
        # engines with read_ints bring counts back without a copy engine, so
        # the read does not wait behind a download on another stream
        reader = getattr(self.engine, "read_ints", None)
        return reader(t) if reader is not None else t.tolist()

    def _over_capacity(self, T: int, recv_rows: torch.Tensor) -> torch.Tensor:
        """[1] int64 on the device: 1 when some rank's local tokens plus
        received rows exceed its engine's capacity (MAX over the ranks, so
        every rank reads the same verdict with its counts)."""
        limit = self.max_rows if self.max_rows is not None else 1 << 62
        flag = (recv_rows.sum() + T > limit).to(torch.int64).reshape(1)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.group)
        return flag

    @staticmethod
    def _raise_over_capacity(flag: int) -> None:
        if flag:
            # every rank raises here, after the same collectives
            raise ValueError("GLM5X_EP_ROWS_EXCEED_MAX_TOKENS")

    def __call__(self, hidden: torch.Tensor) -> torch.Tensor:
        H = self.hidden_size
        x = hidden.reshape(-1, H).to(torch.bfloat16).contiguous()
        T = x.shape[0]
        evs = [] if self._timing else None
        self._mark(evs)
        ids, w = self.engine.route(x)
        self._mark(evs)
        if self.fp4_dispatch:
            out = self._forward_fp4(x, ids, w, evs)
            return out.reshape(*hidden.shape[:-1], H)
        # counts first: one host read for both directions (the split sizes)
        mask = self._dest_mask(ids)
        send_counts = mask.sum(dim=0)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts.contiguous(), group=self.group)
        over = self._over_capacity(T, recv_counts)
        counts = self._host_ints(torch.cat([send_counts, recv_counts, over]))
        self._raise_over_capacity(counts[2 * self.world])
        sc, rc = counts[:self.world], counts[self.world:2 * self.world]
        self.last_counts = (sc, rc)
        R = sum(rc)
        d_idx, t_idx = self._pairs(mask, sum(sc))
        # per pair: k masked ids and k weights (as raw 32-bit words) in one row
        sel = ids[t_idx]
        meta = torch.cat([torch.where(sel.long() // self.per == d_idx[:, None], sel,
                                      torch.full_like(sel, -1)),
                          w[t_idx].view(torch.int32)], dim=1).contiguous()
        send_rows = x[t_idx].contiguous()
        # local tokens first (shared expert), then the received rows; the
        # local rows are copied by a kernel (x * 1 is exact), not a copy engine
        rows = torch.empty((T + R, H), dtype=torch.bfloat16, device=x.device)
        torch.mul(x, 1, out=rows[:T])
        dist.all_to_all_single(rows[T:], send_rows, rc, sc, group=self.group)
        rmeta = torch.empty((T + R, 2 * self.top_k), dtype=torch.int32, device=x.device)
        rmeta[:T, :self.top_k] = -1
        rmeta[:T, self.top_k:] = 0
        dist.all_to_all_single(rmeta[T:], meta, rc, sc, group=self.group)
        rids = rmeta[:, :self.top_k]
        rw = rmeta[:, self.top_k:].view(torch.float32)
        self._mark(evs)
        y = self.engine.forward_expert_rows(rows, rids, rw, shared_rows=T)
        self._mark(evs)
        # partial sums travel back as BF16 (each is a sum of BF16 expert
        # outputs already; rounding it once more costs 2^-9 relative)
        back = torch.empty((t_idx.numel(), H), dtype=torch.bfloat16, device=x.device)
        dist.all_to_all_single(back, y[T:].to(torch.bfloat16), sc, rc, group=self.group)
        out = y[:T]
        # pos[t, d] = row of pair (t, d) in `back`, -1 if the token sent nothing
        # to rank d; partial sums are added in destination order
        pos = torch.full((T, self.world), -1, dtype=torch.int32, device=x.device)
        pos[t_idx, d_idx] = torch.arange(t_idx.numel(), dtype=torch.int32, device=x.device)
        self.combine(back, pos, out)
        self._mark(evs)
        if evs is not None:
            self._pending.append(evs)
        return out.reshape(*hidden.shape[:-1], H)

    def _forward_fp4(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, evs):
        T, H, k, W = x.shape[0], self.hidden_size, self.top_k, self.world
        dev = x.device
        if T:
            amax = self.engine.slab_amax(x, ids)
        else:  # no local tokens: nothing of this rank's in any slab
            amax = torch.zeros(self.num_experts, dtype=torch.float32, device=dev)
        dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)
        # (token, slot) pairs with an expert, by destination rank, then token, then slot
        flat_ids = ids.reshape(-1).long()
        valid = flat_ids >= 0
        dest = torch.where(valid, flat_ids // self.per, torch.full_like(flat_ids, W))
        n_flat = flat_ids.numel()
        order = torch.argsort(dest * n_flat + torch.arange(n_flat, device=dev))
        # per destination: rows (token, expert pairs) and distinct tokens; the
        # receiver's rows and row groups per source come back in one exchange
        mask = self._dest_mask(ids)
        # (a scatter-add count: CUDA bincount reads its input's maximum back)
        rows_per = torch.zeros(W + 1, dtype=torch.int64, device=dev)
        rows_per.scatter_add_(0, dest, torch.ones_like(dest))
        send = torch.stack([rows_per[:W], mask.sum(dim=0)], dim=1)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send.contiguous(), group=self.group)
        over = self._over_capacity(T, recv[:, 0])
        counts = self._host_ints(torch.cat([send.t().reshape(-1), recv.t().reshape(-1), over]))
        self._raise_over_capacity(counts[4 * W])
        sc, tc, rc, gcount = (counts[0:W], counts[W:2 * W], counts[2 * W:3 * W],
                              counts[3 * W:4 * W])
        n_pairs, R, G = sum(sc), sum(rc), sum(gcount)
        order = order[:n_pairs]
        pair_tok = (order // k).to(torch.int32)
        pair_exp = flat_ids[order].to(torch.int32)
        pair_w = w.reshape(-1)[order].float()
        if n_pairs:
            packed, scales = self.engine.quantize_rows(x, pair_tok, pair_exp, amax)
        else:
            packed = torch.empty((0, H // 2), dtype=torch.uint8, device=dev)
            scales = torch.empty((0, H // 16), dtype=torch.uint8, device=dev)
        meta = torch.stack([pair_exp, pair_w.view(torch.int32), pair_tok], dim=1).contiguous()
        rpacked = torch.empty((R, H // 2), dtype=torch.uint8, device=dev)
        rscales = torch.empty((R, H // 16), dtype=torch.uint8, device=dev)
        rmeta = torch.empty((R, 3), dtype=torch.int32, device=dev)
        dist.all_to_all_single(rpacked, packed, rc, sc, group=self.group)
        dist.all_to_all_single(rscales, scales, rc, sc, group=self.group)
        dist.all_to_all_single(rmeta, meta, rc, sc, group=self.group)
        # groups: consecutive received rows of one source token (source rank
        # order); G, known from the exchange, sizes them without a read-back
        src = torch.repeat_interleave(torch.arange(W, device=dev), recv[:, 0], output_size=R)
        tok = rmeta[:, 2]
        new = torch.ones(R, dtype=torch.bool, device=dev)
        if R > 1:
            new[1:] = (src[1:] != src[:-1]) | (tok[1:] != tok[:-1])
        gid = torch.cumsum(new.long(), 0) - 1
        first = torch.empty(G + 1, dtype=torch.int64, device=dev)
        first.scatter_(0, torch.where(new, gid, torch.full_like(gid, G)),
                       torch.arange(R, device=dev))
        first = first[:G]
        group_rows = torch.full((G, k), -1, dtype=torch.int32, device=dev)
        if R:
            slot = torch.arange(R, device=dev) - first[gid]
            group_rows[gid, slot] = torch.arange(R, dtype=torch.int32, device=dev)
        self.last_counts = (sc, rc)
        self._mark(evs)
        if T or R:
            out, out_groups = self.engine.forward_quantized_rows(
                x, rpacked, rscales, rmeta[:, 0], rmeta[:, 1].view(torch.float32), amax,
                group_rows)
        else:  # nothing local, nothing received: no engine work this step
            out = torch.empty((0, H), dtype=torch.float32, device=dev)
            out_groups = torch.empty((0, H), dtype=torch.float32, device=dev)
        self._mark(evs)
        # one partial sum per (token, destination) returns, as in the BF16 dispatch
        d_idx, t_idx = self._pairs(mask, sum(tc))
        back = torch.empty((t_idx.numel(), H), dtype=torch.bfloat16, device=dev)
        dist.all_to_all_single(back, out_groups.to(torch.bfloat16), tc, gcount,
                               group=self.group)
        pos = torch.full((T, W), -1, dtype=torch.int32, device=dev)
        pos[t_idx, d_idx] = torch.arange(t_idx.numel(), dtype=torch.int32, device=dev)
        self.combine(back, pos, out)
        self._mark(evs)
        if evs is not None:
            self._pending.append(evs)
        return out

    @staticmethod
    def combine(rows: torch.Tensor, pos: torch.Tensor, out: torch.Tensor) -> None:
        """out[t] += sum_d rows[pos[t, d]] (pos < 0 skipped), FP32, fixed order.
        Device tensors go through glm5x_combine_rows; the host loop serves
        engines that return host tensors (the CPU stand-in of the gloo tests),
        it is never a substitute for the device kernel."""
        if out.shape[0] == 0:  # a rank with no local tokens has nothing to add
            return
        if out.is_cuda:
            from . import _native as N
            N.check(N.lib().glm5x_combine_rows(
                rows.data_ptr(), pos.data_ptr(), out.shape[0], pos.shape[1], out.shape[1],
                out.data_ptr(), 1, N.stream_arg(torch.cuda.current_stream().cuda_stream)))
            return
        for d in range(pos.shape[1]):
            sel = pos[:, d] >= 0
            out[sel] += rows[pos[sel, d].long()].float()

    def count_local_assignments(self, rows_ids: torch.Tensor, begin: int) -> int:
        """Held (row, slot) assignments among dispatched rows (synchronizes)."""
        return int(((rows_ids >= begin) & (rows_ids < begin + self.per)).sum().item())


def expert_range(rank: int, world: int, num_experts: int) -> tuple[int, int]:
    """(first expert, count) held by `rank`."""
    per = num_experts // world
    return rank * per, per


def bias_balanced_order(bias, world: int) -> list[int]:
    """Expert placement for expert parallelism taken from the router's
    correction bias: renumbered expert j (held by rank j // (E / world), as
    `expert_range` assigns) is original expert ``order[j]``.

    Experts are dealt to the ranks in bias order, largest first, in a snake
    (ranks 0 .. W-1, then W-1 .. 0, ...), so every rank holds experts of
    every bias level. The correction bias is what tilts the top-k towards
    some experts, so the ranks' loads even out: config 5 at 8 ranks puts
    1.01x the mean routed rows on the busiest rank, against 1.20x with
    contiguous ranges of original ids. Loading original expert ``order[j]``
    as expert j and setting the router with its rows and bias permuted by
    ``order`` computes the same layer (the top-k picks the same experts under
    their new numbers; only exact score ties, broken by the lower id, could
    pick differently). Needs E divisible by world."""
    b = [float(v) for v in bias]
    num_experts = len(b)
    if world < 1 or num_experts % world:
        raise ValueError("GLM5X_EP_WORLD: experts must divide evenly over the ranks")
    ranked = sorted(range(num_experts), key=lambda e: (-b[e], e))
    slots: list[list[int]] = [[] for _ in range(world)]
    for i, e in enumerate(ranked):
        rnd, pos = divmod(i, world)
        slots[pos if rnd % 2 == 0 else world - 1 - pos].append(e)
    return [e for r in range(world) for e in slots[r]]
