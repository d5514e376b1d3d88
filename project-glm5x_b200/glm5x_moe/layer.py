"""The MoE sublayer engine, mirroring the reference's layer interface.

``GLM5XMoELayer`` takes the arguments of ``GLM5XLayer10MoEReference``
(reference/glm5x_ref/layer10_moe.py:349-374) that matter for the routed-expert
path (router weight, correction bias, top_k, routed_scaling_factor, a shared
expert, NVFP4 experts) and returns a ``GLM5XMoEForward``-shaped result
(output, router_logits, topk_indices, topk_weights). All work runs in
libglm5x_moe.so on one CUDA device.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Mapping

import torch

from . import _native as N
from .nvfp4 import GLM5XMXFP4Weight, GLM5XNVFP4Weight


@dataclass(frozen=True)
class GLM5XMoEForward:
    """(reference/glm5x_ref/layer10_moe.py:93-101, minus loaded_experts)"""

    output: torch.Tensor
    router_logits: torch.Tensor | None
    topk_indices: torch.Tensor | None
    topk_weights: torch.Tensor | None


@dataclass(frozen=True)
class NVFP4Expert:
    """gate/up [I, H] and down [H, I] NVFP4 projections of one expert."""

    gate_proj: GLM5XNVFP4Weight
    up_proj: GLM5XNVFP4Weight
    down_proj: GLM5XNVFP4Weight


@dataclass(frozen=True)
class MXFP4Expert:
    """gate/up [I, H] and down [H, I] MXFP4 projections of one expert."""

    gate_proj: GLM5XMXFP4Weight
    up_proj: GLM5XMXFP4Weight
    down_proj: GLM5XMXFP4Weight


def _stream() -> ctypes.c_void_p:
    return N.stream_arg(torch.cuda.current_stream().cuda_stream)


class GLM5XMoELayer:
    """Routed-expert MoE sublayer on a B200 (sm_100) through the C ABI."""

    def __init__(self, *, hidden_size: int = 6144, intermediate_size: int = 2048,
                 num_experts: int = 256, top_k: int = 8, routed_scaling_factor: float = 2.5,
                 has_shared: bool = True, max_tokens: int = 8192, device: int = 0,
                 precision: str = "nvfp4", expert_begin: int = 0,
                 expert_count: int | None = None) -> None:
        if precision not in {"nvfp4", "mxfp4"}:
            raise ValueError("GLM5X_INVALID_EXPERT_PRECISION")
        if not isinstance(top_k, int) or not 0 < top_k <= num_experts:
            raise ValueError("GLM5X_INVALID_TOP_K")
        if routed_scaling_factor <= 0:
            raise ValueError("GLM5X_INVALID_ROUTED_SCALE")
        cfg = N.MoeConfig(hidden_size, intermediate_size, num_experts, top_k,
                          1 if has_shared else 0, float(routed_scaling_factor),
                          N.PRECISION_NVFP4 if precision == "nvfp4" else N.PRECISION_MXFP4,
                          max_tokens, expert_begin,
                          expert_count if expert_count is not None else num_experts)
        handle = ctypes.c_void_p()
        N.check(N.lib().glm5x_moe_create(ctypes.byref(cfg), device, ctypes.byref(handle)))
        self._h = handle
        self.device = torch.device("cuda", device)
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.has_shared = has_shared
        self.max_tokens = max_tokens
        self._in_flight: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    @classmethod
    def _borrow(cls, handle: int, *, hidden_size: int, intermediate_size: int, num_experts: int,
                top_k: int, has_shared: bool, max_tokens: int, device: int) -> "GLM5XMoELayer":
        """A view of an engine another object owns (the engine of an
        expert-parallel rank): weights and router go through it; close()
        leaves the engine to its owner."""
        self = cls.__new__(cls)
        self._h = ctypes.c_void_p(handle)
        self._owned = False
        self.device = torch.device("cuda", device)
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.has_shared = has_shared
        self.max_tokens = max_tokens
        self._in_flight = {}
        return self

    def close(self) -> None:
        if getattr(self, "_h", None) and not getattr(self, "_owned", True):
            self._h = None
            return
        if getattr(self, "_h", None):
            # destroy synchronizes every stream before the host buffers go
            N.lib().glm5x_moe_destroy(self._h)
            self._h = None
            self._in_flight = {}

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------ weights
    def set_router(self, router_weight: torch.Tensor, correction_bias: torch.Tensor) -> None:
        w = router_weight.detach().to(device="cpu", dtype=torch.bfloat16).contiguous()
        b = correction_bias.detach().to(device="cpu", dtype=torch.float32).contiguous()
        if tuple(w.shape) != (self.num_experts, self.hidden_size):
            raise ValueError("GLM5X_ROUTER_WEIGHT_SHAPE")
        if tuple(b.shape) != (self.num_experts,):
            raise ValueError("GLM5X_ROUTER_BIAS_SHAPE")
        N.check(N.lib().glm5x_moe_set_router(self._h, w.data_ptr(), b.data_ptr()), self._h)

    def load_expert(self, expert_id: int, expert: NVFP4Expert | MXFP4Expert) -> None:
        """Admit one NVFP4 or MXFP4 expert held in device tensors (expert_id -1
        = shared); the format must match the layer's precision."""
        g, u, d = expert.gate_proj.matrix(), expert.up_proj.matrix(), expert.down_proj.matrix()
        fn = (N.lib().glm5x_moe_load_expert_mxfp4_device if isinstance(expert, MXFP4Expert)
              else N.lib().glm5x_moe_load_expert_nvfp4_device)
        with torch.cuda.device(self.device):
            torch.cuda.current_stream().synchronize()
            N.check(fn(self._h, expert_id, ctypes.byref(g), ctypes.byref(u), ctypes.byref(d)),
                    self._h)

    def load_expert_bf16(self, expert_id: int, gate_proj: torch.Tensor, up_proj: torch.Tensor,
                         down_proj: torch.Tensor, *, scale_mode: str = "mse") -> None:
        """Admit a float expert (gate/up [I, H], down [H, I]) packed on the
        device at admission: NVFP4 layers pack each projection with the
        reference's quantize_nvfp4_weight semantics (_quantize_expert_nvfp4,
        layer10_moe.py:603-619), MXFP4 layers with encode_mxfp4 (group 32)."""
        mode = {"max_abs": N.SCALE_MAX_ABS, "mse": N.SCALE_MSE}[scale_mode]
        mats = [t.detach().to(dtype=torch.bfloat16).contiguous()
                for t in (gate_proj, up_proj, down_proj)]
        I, H = self.intermediate_size, self.hidden_size
        if (tuple(mats[0].shape) != (I, H) or tuple(mats[1].shape) != (I, H)
                or tuple(mats[2].shape) != (H, I)):
            raise ValueError("GLM5X_EXPERT_WEIGHT_SHAPE_MISMATCH")
        on_device = all(m.is_cuda for m in mats)
        if on_device:
            mats = [m.to(self.device) for m in mats]
        else:
            mats = [m.cpu() for m in mats]
        fn = (N.lib().glm5x_moe_load_expert_bf16_device if on_device
              else N.lib().glm5x_moe_load_expert_bf16)
        with torch.cuda.device(self.device):
            torch.cuda.current_stream().synchronize()
            N.check(fn(self._h, expert_id, mats[0].data_ptr(), mats[1].data_ptr(),
                       mats[2].data_ptr(), mode), self._h)

    def load_expert_k3x(self, expert_id: int, k3x_file, prefix: str) -> None:
        """Admit expert ``expert_id`` (-1 = shared) from the MXFP4 records
        ``<prefix>.gate / .up / .down`` of an open ``k3x.K3xFile`` (e.g.
        prefix "model.layers.1.feed_forward.experts.3"); MXFP4 layers only."""
        N.check(N.lib().glm5x_moe_load_expert_k3x(self._h, expert_id, k3x_file.handle,
                                                  prefix.encode()), self._h)

    def load_sidecar(self, expert_id: int, path: str) -> None:
        N.check(N.lib().glm5x_moe_load_sidecar(self._h, expert_id, str(path).encode()), self._h)

    # ------------------------------------------------------------ forward
    def __call__(self, hidden_states: torch.Tensor, *, want_routing: bool = True
                 ) -> GLM5XMoEForward:
        if hidden_states.ndim < 2 or hidden_states.shape[-1] != self.hidden_size:
            raise ValueError("GLM5X_MOE_HIDDEN_SHAPE")
        shape = hidden_states.shape
        flat = hidden_states.reshape(-1, self.hidden_size).to(torch.bfloat16).contiguous()
        if flat.device != self.device:
            raise ValueError("GLM5X_MOE_DEVICE_MISMATCH")
        T = flat.shape[0]
        out = torch.empty((T, self.hidden_size), dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            N.check(N.lib().glm5x_moe_forward(self._h, flat.data_ptr(), T, out.data_ptr(),
                                              _stream()), self._h)
            if not want_routing:
                return GLM5XMoEForward(out.reshape(shape), None, None, None)
            torch.cuda.current_stream().synchronize()
            ids = torch.empty((T, self.top_k), dtype=torch.int32)
            w = torch.empty((T, self.top_k), dtype=torch.float32)
            logits = torch.empty((T, self.num_experts), dtype=torch.float32)
            N.check(N.lib().glm5x_moe_last_routing(self._h, ids.data_ptr(), w.data_ptr(),
                                                   logits.data_ptr(), T), self._h)
            N.check(N.lib().glm5x_moe_check(self._h), self._h)
        return GLM5XMoEForward(
            output=out.reshape(shape),
            router_logits=logits.reshape(*shape[:-1], self.num_experts),
            topk_indices=ids.reshape(*shape[:-1], self.top_k),
            topk_weights=w.reshape(*shape[:-1], self.top_k))

    def forward_routed(self, hidden: torch.Tensor, ids: torch.Tensor,
                       weights: torch.Tensor) -> torch.Tensor:
        """Expert path with caller-supplied routing (ids [T,k] int32,
        weights [T,k] fp32, device tensors)."""
        flat = hidden.reshape(-1, self.hidden_size).to(torch.bfloat16).contiguous()
        T = flat.shape[0]
        ids = ids.to(device=self.device, dtype=torch.int32).contiguous()
        weights = weights.to(device=self.device, dtype=torch.float32).contiguous()
        if tuple(ids.shape) != (T, self.top_k) or tuple(weights.shape) != (T, self.top_k):
            raise ValueError("GLM5X_ROUTING_SHAPE")
        out = torch.empty((T, self.hidden_size), dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            N.check(N.lib().glm5x_moe_forward_routed(self._h, flat.data_ptr(), T, ids.data_ptr(),
                                                     weights.data_ptr(), out.data_ptr(),
                                                     _stream()), self._h)
        return out

    def route(self, hidden: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Router only: (ids [T, k] int32, weights [T, k] fp32) on the device."""
        flat = hidden.reshape(-1, self.hidden_size).to(torch.bfloat16).contiguous()
        T = flat.shape[0]
        ids = torch.empty((T, self.top_k), dtype=torch.int32, device=self.device)
        w = torch.empty((T, self.top_k), dtype=torch.float32, device=self.device)
        if T == 0:  # an expert-parallel rank with no local tokens this step
            return ids, w
        with torch.cuda.device(self.device):
            N.check(N.lib().glm5x_moe_route(self._h, flat.data_ptr(), T, ids.data_ptr(),
                                            w.data_ptr(), None, _stream()), self._h)
        return ids, w

    def forward_expert_rows(self, rows: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                            shared_rows: int = 0) -> torch.Tensor:
        """Experts held by this engine over dispatched rows: ids are global
        expert ids (others / -1 skipped); rows < shared_rows also take the
        shared expert. Returns FP32 [R, H]."""
        flat = rows.reshape(-1, self.hidden_size).to(torch.bfloat16).contiguous()
        R = flat.shape[0]
        out = torch.empty((R, self.hidden_size), dtype=torch.float32, device=self.device)
        if R == 0:
            return out
        ids = ids.to(device=self.device, dtype=torch.int32).contiguous()
        weights = weights.to(device=self.device, dtype=torch.float32).contiguous()
        if tuple(ids.shape) != (R, self.top_k) or tuple(weights.shape) != (R, self.top_k):
            raise ValueError("GLM5X_ROUTING_SHAPE")
        with torch.cuda.device(self.device):
            N.check(N.lib().glm5x_moe_forward_expert_rows(
                self._h, flat.data_ptr(), R, ids.data_ptr(), weights.data_ptr(), shared_rows,
                out.data_ptr(), _stream()), self._h)
        return out

    def forward_host(self, hidden_bf16_host: torch.Tensor, out_host: torch.Tensor) -> None:
        """Host buffers in/out: H2D copy, forward, D2H copy, synchronize."""
        T = hidden_bf16_host.shape[0]
        N.check(N.lib().glm5x_moe_forward_host(self._h, hidden_bf16_host.data_ptr(), T,
                                               out_host.data_ptr()), self._h)

    def submit_host(self, hidden_bf16_host: torch.Tensor, out_host: torch.Tensor) -> int:
        """Pipelined host forward: enqueues upload, forward and download and
        returns a ticket for wait_host(). Both tensors are held until then."""
        T = hidden_bf16_host.shape[0]
        if (hidden_bf16_host.device.type != "cpu" or out_host.device.type != "cpu"
                or hidden_bf16_host.dtype != torch.bfloat16 or out_host.dtype != torch.float32
                or not hidden_bf16_host.is_contiguous() or not out_host.is_contiguous()
                or tuple(hidden_bf16_host.shape) != (T, self.hidden_size)
                or tuple(out_host.shape) != (T, self.hidden_size)):
            raise ValueError("GLM5X_HOST_BUFFERS")
        ticket = ctypes.c_int64()
        N.check(N.lib().glm5x_moe_submit_host(self._h, hidden_bf16_host.data_ptr(), T,
                                              out_host.data_ptr(), ctypes.byref(ticket)),
                self._h)
        self._in_flight[ticket.value] = (hidden_bf16_host, out_host)
        return ticket.value

    def wait_host(self, ticket: int) -> None:
        """Waits for a submit_host() ticket; raises its forward's device error."""
        try:
            N.check(N.lib().glm5x_moe_wait_host(self._h, ticket), self._h)
        finally:
            self._in_flight.pop(ticket, None)

    def read_ints(self, t: torch.Tensor) -> list[int]:
        """A small device int64 tensor's values on the host, after the work on
        the current stream, without a copy-engine transfer."""
        src = t.reshape(-1).to(dtype=torch.int64).contiguous()
        if src.device.type != "cuda":
            return src.tolist()
        n = src.numel()
        out = (ctypes.c_int64 * max(n, 1))()
        with torch.cuda.device(self.device):
            N.check(N.lib().glm5x_moe_read_ints(self._h, src.data_ptr(), n,
                                                ctypes.addressof(out), _stream()), self._h)
        return list(out[:n])

    def check(self) -> None:
        N.check(N.lib().glm5x_moe_check(self._h), self._h)

    def debug_buffer(self, which: int) -> tuple[int, int]:
        ptr = ctypes.c_void_p()
        size = ctypes.c_size_t()
        N.check(N.lib().glm5x_moe_debug_buffer(self._h, which, ctypes.byref(ptr),
                                               ctypes.byref(size)), self._h)
        return int(ptr.value or 0), int(size.value)

    def debug_tensor(self, which: int, dtype: torch.dtype, count: int) -> torch.Tensor:
        """Copy the first `count` elements of an internal device buffer."""
        esz = torch.tensor([], dtype=dtype).element_size()
        out = torch.empty(count, dtype=dtype, device=self.device)
        with torch.cuda.device(self.device):
            torch.cuda.current_stream().synchronize()
            N.check(N.lib().glm5x_moe_debug_copy(self._h, which, out.data_ptr(), count * esz),
                    self._h)
        return out

    def set_tile_n(self, bn: int) -> None:
        """Force the expert GEMMs' token tile (32/64/128/256), 0 = automatic."""
        N.check(N.lib().glm5x_moe_set_tile_n(self._h, bn), self._h)

    def set_pair_mma(self, enable: bool) -> None:
        """256-row token tiles on CTA pairs (default) or single CTAs."""
        N.check(N.lib().glm5x_moe_set_pair_mma(self._h, 1 if enable else 0), self._h)

    # ---------------------------------------------- expert-parallel FP4 dispatch
    def slab_amax(self, hidden: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        """Per-expert max |x| of this rank's tokens routed to each expert
        (FP32 [num_experts], device); reduce it with MAX over the ranks."""
        flat = hidden.reshape(-1, self.hidden_size).to(torch.bfloat16).contiguous()
        ids = ids.to(device=self.device, dtype=torch.int32).contiguous()
        amax = torch.empty(self.num_experts, dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            N.check(N.lib().glm5x_moe_slab_amax(self._h, flat.data_ptr(), flat.shape[0],
                                                ids.data_ptr(), amax.data_ptr(), _stream()),
                    self._h)
        return amax

    def quantize_rows(self, hidden: torch.Tensor, row_token: torch.Tensor,
                      row_expert: torch.Tensor, amax: torch.Tensor):
        """NVFP4 rows to send: token row_token[r] quantized for expert
        row_expert[r] with that expert's reduced slab scale. Returns
        (packed uint8 [n, H/2], scales uint8 [n, H/16] row-major E4M3)."""
        flat = hidden.reshape(-1, self.hidden_size).to(torch.bfloat16).contiguous()
        tok = row_token.to(device=self.device, dtype=torch.int32).contiguous()
        exp = row_expert.to(device=self.device, dtype=torch.int32).contiguous()
        n = tok.numel()
        H = self.hidden_size
        packed = torch.empty((n, H // 2), dtype=torch.uint8, device=self.device)
        scales = torch.empty((n, H // 16), dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            N.check(N.lib().glm5x_moe_quantize_rows(
                self._h, flat.data_ptr(), flat.shape[0], tok.data_ptr(), exp.data_ptr(), n,
                amax.data_ptr(), packed.data_ptr(), scales.data_ptr(), _stream()), self._h)
        return packed, scales

    def forward_quantized_rows(self, hidden: torch.Tensor, packed: torch.Tensor,
                               scales: torch.Tensor, row_expert: torch.Tensor,
                               row_weight: torch.Tensor, amax: torch.Tensor,
                               group_rows: torch.Tensor):
        """The local tokens through the shared expert and the received NVFP4
        rows through their held experts. Returns (out_local FP32 [T, H],
        out_groups FP32 [G, H]) with out_groups[g] = the sum of the weighted
        expert rows of received rows group_rows[g, :] (-1 = none)."""
        flat = hidden.reshape(-1, self.hidden_size).to(torch.bfloat16).contiguous()
        T, H = flat.shape[0], self.hidden_size
        exp = row_expert.to(device=self.device, dtype=torch.int32).contiguous()
        wts = row_weight.to(device=self.device, dtype=torch.float32).contiguous()
        grp = group_rows.to(device=self.device, dtype=torch.int32).contiguous()
        R = exp.numel()
        G, slots = grp.shape
        out_local = torch.empty((T, H), dtype=torch.float32, device=self.device)
        out_groups = torch.empty((G, H), dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            N.check(N.lib().glm5x_moe_forward_quantized_rows(
                self._h, flat.data_ptr() if T else None, T, packed.data_ptr() if R else None,
                scales.data_ptr() if R else None, exp.data_ptr() if R else None,
                wts.data_ptr() if R else None, R, amax.data_ptr(),
                out_local.data_ptr() if T else None,
                grp.data_ptr() if G else None, G, max(slots, 1),
                out_groups.data_ptr() if G else None, _stream()), self._h)
        return out_local, out_groups

    def set_routing_policy(self, config, collect_diagnostics: bool = False) -> None:
        """select_routing policy of the router (a routing.RoutingPolicyConfig:
        natural, fixed or adaptive Top-K with a quality floor). Fixed and
        adaptive leave id -1 / weight 0 in the slots past each token's K;
        ``collect_diagnostics`` keeps the per-token decision scalars in
        natural mode too."""
        pol = config.to_c(collect_diagnostics)
        N.check(N.lib().glm5x_moe_set_routing_policy(self._h, ctypes.byref(pol)), self._h)

    def routing_stats(self) -> dict:
        """Counters of the last router pass with diagnostics (the reference
        session's routing_* fields): decisions, selected_experts,
        quality_escalated_decisions and the entropy / mass / confidence sums."""
        st = N.RoutingStats()
        N.check(N.lib().glm5x_moe_routing_stats(self._h, ctypes.byref(st)), self._h)
        return {name: getattr(st, name) for name, _ in N.RoutingStats._fields_}

    def routing_decisions(self, tokens: int):
        """Per-token decisions of the last router pass over ``tokens`` tokens
        (CPU tensors): (sel [T, 2] int32 = selected K, escalated; diag [T, 4]
        = normalized entropy, effective support, selected mass, confidence)."""
        sel = torch.empty((tokens, 2), dtype=torch.int32)
        diag = torch.empty((tokens, 4), dtype=torch.float32)
        N.check(N.lib().glm5x_moe_routing_decisions(self._h, tokens, sel.data_ptr(),
                                                    diag.data_ptr()), self._h)
        return sel, diag

    def set_pair_wide_stages(self, enable: bool) -> None:
        """CTA-pair GEMMs with 512-K pipeline stages (or 256-K)."""
        N.check(N.lib().glm5x_moe_set_pair_wide_stages(self._h, 1 if enable else 0), self._h)

    def set_pair_tile_order(self, up_group: int, down_group: int) -> None:
        """Tile order of the CTA-pair GEMMs: 0 = segment-major, g > 0 =
        groups of about g token tiles, each run weight-tile-major."""
        N.check(N.lib().glm5x_moe_set_pair_tile_order(self._h, int(up_group), int(down_group)),
                self._h)

    def set_weight_tile_rows(self, rows: int) -> None:
        """Weight rows per tile for narrow token tiles: 128, or 256 as two
        halves per stage (small batches)."""
        N.check(N.lib().glm5x_moe_set_weight_tile_rows(self._h, rows), self._h)

    def set_down_tile_n(self, bn: int) -> None:
        """Weight-major down projection token tile (128/256, 0 = gate/up's)."""
        N.check(N.lib().glm5x_moe_set_down_tile_n(self._h, bn), self._h)

    def set_token_major_down(self, enable: bool) -> None:
        """Token-major down projection for large batches, or weight-major
        tiles (default)."""
        N.check(N.lib().glm5x_moe_set_token_major_down(self._h, 1 if enable else 0), self._h)

    def set_profiling(self, enable: bool) -> None:
        N.check(N.lib().glm5x_moe_set_profiling(self._h, 1 if enable else 0), self._h)

    def phase_times(self) -> tuple[dict, int]:
        """(milliseconds per phase accumulated since the last call, forwards)."""
        ms = (ctypes.c_float * N.NUM_PHASES)()
        n = ctypes.c_int32()
        N.check(N.lib().glm5x_moe_phase_times(self._h, ms, ctypes.byref(n)), self._h)
        return {name: float(ms[i]) for i, name in enumerate(N.PHASE_NAMES)}, int(n.value)

    def stream_handle(self) -> int:
        s = ctypes.c_void_p()
        N.check(N.lib().glm5x_moe_get_stream(self._h, ctypes.byref(s)), self._h)
        return int(s.value or 0)

    def stats(self) -> Mapping[str, int]:
        s = N.MoeStats()
        N.check(N.lib().glm5x_moe_get_stats(self._h, ctypes.byref(s)), self._h)
        return {name: int(getattr(s, name)) for name, _ in N.MoeStats._fields_}
