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
   counts go first (all-to-all of int64), then rows, ids and weights
   (all-to-all-v);
3. runs its experts over [local tokens; received rows] in one engine call:
   the local tokens take only the shared expert, the received rows only the
   held routed experts;
4. combine: each received row's weighted sum returns to its source
   (all-to-all-v of FP32 rows), where the partial sums of a token are added
   in destination-rank order onto its shared-expert output.

Everything runs on the caller's current stream; torch.distributed (NCCL on
GPUs) moves the bytes. The engine is any object with route(hidden) ->
(ids, weights) and forward_expert_rows(rows, ids, weights, shared_rows).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class ExpertParallelMoE:
    """Dispatch / expert / combine around one rank's engine."""

    def __init__(self, engine, *, rank: int, world: int, num_experts: int, top_k: int,
                 hidden_size: int, group=None) -> None:
        if num_experts % world:
            raise ValueError("GLM5X_EP_EXPERTS_NOT_DIVISIBLE")
        self.engine = engine
        self.rank = rank
        self.world = world
        self.per = num_experts // world
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.group = group
        self.last_counts: tuple[list[int], list[int]] | None = None

    def plan(self, ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(dest [n], token [n], counts [W]) of the dispatch pairs, ordered by
        destination rank, tokens ascending within a destination."""
        T = ids.shape[0]
        dest = ids.long() // self.per
        mask = torch.zeros((T, self.world), dtype=torch.bool, device=ids.device)
        mask.scatter_(1, dest, True)
        d_idx, t_idx = mask.t().nonzero(as_tuple=True)
        return d_idx, t_idx, mask.sum(dim=0)

    def __call__(self, hidden: torch.Tensor) -> torch.Tensor:
        H = self.hidden_size
        x = hidden.reshape(-1, H).to(torch.bfloat16).contiguous()
        T = x.shape[0]
        ids, w = self.engine.route(x)
        d_idx, t_idx, send_counts = self.plan(ids)
        send_ids = torch.where(ids[t_idx].long() // self.per == d_idx[:, None], ids[t_idx],
                               torch.full_like(ids[t_idx], -1)).contiguous()
        send_w = w[t_idx].contiguous()
        send_rows = x[t_idx].contiguous()
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts.contiguous(), group=self.group)
        sc = send_counts.tolist()
        rc = recv_counts.tolist()
        self.last_counts = (sc, rc)
        R = sum(rc)
        # local tokens first (shared expert), then the received rows
        rows = torch.empty((T + R, H), dtype=torch.bfloat16, device=x.device)
        rows[:T] = x
        dist.all_to_all_single(rows[T:], send_rows, rc, sc, group=self.group)
        rids = torch.full((T + R, self.top_k), -1, dtype=torch.int32, device=x.device)
        rw = torch.zeros((T + R, self.top_k), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(rids[T:], send_ids, rc, sc, group=self.group)
        dist.all_to_all_single(rw[T:], send_w, rc, sc, group=self.group)
        y = self.engine.forward_expert_rows(rows, rids, rw, shared_rows=T)
        back = torch.empty((t_idx.numel(), H), dtype=torch.float32, device=x.device)
        dist.all_to_all_single(back, y[T:].contiguous(), sc, rc, group=self.group)
        out = y[:T]
        off = 0
        for d in range(self.world):
            n = sc[d]
            if n:
                # one row per token per destination: no index repeats within
                # a call, so the sum order is fixed (destination order)
                out.index_add_(0, t_idx[off:off + n], back[off:off + n])
            off += n
        return out.reshape(*hidden.shape[:-1], H)


def expert_range(rank: int, world: int, num_experts: int) -> tuple[int, int]:
    """(first expert, count) held by `rank`."""
    per = num_experts // world
    return rank * per, per
