"""Greedy verification of speculative draft blocks, many sequences at once.

The reference's expert-major speculative decoding runs each sequence's
[anchor, draft_1 .. draft_n] block through the target as one expert-major
batch (runtime/src/model.cpp:1640-1690; the C5 workload's 2048 sequences x 4
drafts) and commits the matching prefix plus one target token
(verify_greedy_target_block, runtime/src/speculative.cpp:75-113). This
verifies every sequence's block in one device call.
"""
from __future__ import annotations

import torch

from . import _native as N


def verify_greedy_target_blocks(anchors: torch.Tensor, candidates: torch.Tensor,
                                draft_counts: torch.Tensor, targets: torch.Tensor,
                                vocabulary_size: int) -> dict:
    """anchors [S], candidates [S, D], draft_counts [S] (n_s <= D), targets
    [S, D + 1] (the target's argmax after the anchor and after each candidate),
    CUDA tensors. Returns accepted [S] (matching prefix length), committed
    [S, D + 1] (valid up to accepted + 1), all_accepted [S] and status [S]
    (0, 9 = INVALID_EXTENT, 16 = INVALID_STATE, per sequence as the reference
    returns them)."""
    S, D = candidates.shape
    dev = candidates.device
    u32 = lambda t: t.to(device=dev, dtype=torch.int32).contiguous()  # same bits as uint32
    a, c, n, t = u32(anchors), u32(candidates), u32(draft_counts), u32(targets)
    if tuple(t.shape) != (S, D + 1) or a.shape[0] != S or n.shape[0] != S:
        raise ValueError("anchors [S], candidates [S, D], draft_counts [S], targets [S, D + 1]")
    accepted = torch.empty(S, dtype=torch.int32, device=dev)
    committed = torch.zeros((S, D + 1), dtype=torch.int32, device=dev)
    status = torch.empty(S, dtype=torch.int32, device=dev)
    N.check(N.lib().glm5x_verify_greedy_target_blocks(
        a.data_ptr(), c.data_ptr(), n.data_ptr(), t.data_ptr(), S, D, int(vocabulary_size),
        accepted.data_ptr(), committed.data_ptr(), status.data_ptr(),
        N.stream_arg(torch.cuda.current_stream(dev).cuda_stream)))
    return {"accepted": accepted, "committed": committed,
            "all_accepted": (accepted == n) & (status == 0), "status": status}
