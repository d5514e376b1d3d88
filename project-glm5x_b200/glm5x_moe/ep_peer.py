"""Expert parallelism with the token exchange in the library's own kernels
over NVLink peer memory (glm5x_moe_ep_*; see csrc/ep_peer.cu).

The multi-GPU form of the reference's single-process expert path
(layer10_moe.py:791-847 + 954-961), like ep.py, but with no collective in a
forward: each rank maps every peer's memory once (CUDA IPC handles gathered
with torch.distributed at construction), then stores its token rows straight
into the ranks that hold their experts and pulls the weighted partial sums
back, all in stream order and without a host read. The output equals ep.py's
NCCL all-to-all path bit for bit.

    ep = PeerExpertParallelMoE(rank=r, world=W, max_local_tokens=8192, ...)
    ep.engine.set_router(router, bias); ep.engine.load_expert(e, expert)  # held e only
    out = ep(hidden)          # [T, H] FP32 on this rank's GPU
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as N
from .layer import GLM5XMoELayer


class PeerExpertParallelMoE:
    """One rank of the peer-memory expert-parallel layer."""

    def __init__(self, *, rank: int, world: int, max_local_tokens: int, hidden_size: int = 6144,
                 intermediate_size: int = 2048, num_experts: int = 256, top_k: int = 8,
                 routed_scaling_factor: float = 2.5, precision: str = "nvfp4", device: int = 0,
                 group=None) -> None:
        if num_experts % world:
            raise ValueError("GLM5X_EP_EXPERTS_NOT_DIVISIBLE")
        cfg = N.MoeConfig(hidden_size, intermediate_size, num_experts, top_k, 1,
                          float(routed_scaling_factor),
                          N.PRECISION_NVFP4 if precision == "nvfp4" else N.PRECISION_MXFP4,
                          max_local_tokens, 0, num_experts)
        h = ctypes.c_void_p()
        N.check(N.lib().glm5x_moe_ep_create(ctypes.byref(cfg), device, rank, world,
                                            max_local_tokens, ctypes.byref(h)))
        self._h = h
        self.rank, self.world = rank, world
        self.device = torch.device("cuda", device)
        self.hidden_size = hidden_size
        self.max_local_tokens = max_local_tokens
        self.per = num_experts // world
        try:
            own = (ctypes.c_uint8 * N.EP_HANDLE_BYTES)()
            self._check(N.lib().glm5x_moe_ep_handle(h, own))
            handles = self._gather(bytes(own), group)
            buf = (ctypes.c_uint8 * len(handles)).from_buffer_copy(handles)
            self._check(N.lib().glm5x_moe_ep_connect(h, buf))
        except Exception:
            N.lib().glm5x_moe_ep_destroy(h)
            self._h = None
            raise
        self.engine = GLM5XMoELayer._borrow(
            N.lib().glm5x_moe_ep_engine(h), hidden_size=hidden_size,
            intermediate_size=intermediate_size, num_experts=num_experts, top_k=top_k,
            has_shared=True, max_tokens=max_local_tokens * (world + 1), device=device)

    def _gather(self, own: bytes, group) -> bytes:
        """Every rank's handle, in rank order (torch.distributed; nothing to
        exchange with one rank)."""
        if self.world == 1:
            return own
        t = torch.tensor(list(own), dtype=torch.uint8)
        if dist.get_backend(group) == "nccl":
            t = t.to(self.device)
        out = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(out, t, group=group)
        return b"".join(bytes(o.cpu().tolist()) for o in out)

    def _check(self, status: int) -> None:
        if status != 0:
            msg = N.lib().glm5x_moe_ep_error_message(self._h) if self._h else b""
            raise N.Glm5xError(status, (msg or N.lib().glm5x_last_error_message() or b"")
                               .decode(errors="replace"))

    def __call__(self, hidden: torch.Tensor) -> torch.Tensor:
        x = hidden.reshape(-1, self.hidden_size).to(torch.bfloat16).contiguous()
        T = x.shape[0]
        out = torch.empty((T, self.hidden_size), dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            self._check(N.lib().glm5x_moe_ep_forward(
                self._h, x.data_ptr() if T else None, T, out.data_ptr() if T else None,
                N.stream_arg(torch.cuda.current_stream().cuda_stream)))
        return out.reshape(*hidden.shape[:-1], self.hidden_size)

    STAGES = ("route", "exchange", "dispatch", "experts", "combine")

    def set_timing(self, enable: bool) -> None:
        """CUDA events at the stage boundaries of later forwards."""
        self._check(N.lib().glm5x_moe_ep_set_profiling(self._h, 1 if enable else 0))

    def stage_times(self) -> tuple[dict, int]:
        """(milliseconds per stage summed since the last call, forwards):
        route, exchange (plan + counts), dispatch (rows out + wait for every
        source's rows), experts, combine (ready + partial sums pulled back)."""
        ms = (ctypes.c_float * len(self.STAGES))()
        n = ctypes.c_int32()
        self._check(N.lib().glm5x_moe_ep_stage_times(self._h, ms, ctypes.byref(n)))
        return dict(zip(self.STAGES, (float(v) for v in ms))), int(n.value)

    def last_counts(self) -> tuple[list[int], int]:
        """(rows sent to each rank, rows received) of the last forward."""
        sent = (ctypes.c_int64 * self.world)()
        recv = ctypes.c_int64()
        self._check(N.lib().glm5x_moe_ep_last_counts(self._h, sent, ctypes.byref(recv)))
        return list(sent), int(recv.value)

    def check(self) -> None:
        """Synchronizes; raises GLM5X_WAIT_TIMEOUT if a peer did not answer."""
        self._check(N.lib().glm5x_moe_ep_check(self._h))

    def close(self) -> None:
        """Every rank must be done with its last forward (a barrier) first."""
        if getattr(self, "_h", None):
            if hasattr(self, "engine"):
                self.engine.close()
            N.lib().glm5x_moe_ep_destroy(self._h)
            self._h = None

    def __del__(self) -> None:  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass
