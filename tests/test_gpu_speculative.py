"""Batched greedy verification of draft blocks on the GPU (C5's 2048
sequences x 4 drafts and ragged counts) against the oracle, sequence by
sequence: statuses, accepted lengths and committed tokens exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu


def test_batched_verify_matches_oracle():
    from glm5x_moe.speculative import verify_greedy_target_blocks
    rng = np.random.default_rng(5)
    S, D, vocab = 2048, 4, 1000
    anchors = rng.integers(0, vocab, S).astype(np.uint32)
    counts = rng.integers(0, D + 1, S).astype(np.int32)
    cand = rng.integers(0, vocab, (S, D)).astype(np.uint32)
    tgt = np.concatenate([cand, rng.integers(0, vocab, (S, 1))], 1).astype(np.uint32)
    # break the match at a random position in half of the sequences
    brk = rng.integers(0, D + 1, S)
    for s in range(S):
        if s % 2 and brk[s] < D:
            tgt[s, brk[s]] = (cand[s, brk[s]] + 1) % vocab
    # a few invalid proposals / targets
    anchors[3] = vocab
    cand[5, 0] = vocab
    counts[5] = max(counts[5], 1)
    counts[7] = D + 1
    tgt[9, counts[9]] = vocab
    to = lambda a: torch.from_numpy(a.astype(np.int64)).cuda()
    r = verify_greedy_target_blocks(to(anchors), to(cand), to(counts), to(tgt), vocab)
    st, acc = r["status"].cpu().numpy(), r["accepted"].cpu().numpy()
    com = r["committed"].cpu().numpy().astype(np.uint32)
    for s in range(S):
        n = int(counts[s])
        c_s = cand[s, :n] if n <= D else np.concatenate([cand[s], np.zeros(n - D, np.uint32)])
        t_s = tgt[s, :n + 1] if n <= D else np.concatenate([tgt[s], np.zeros(n - D, np.uint32)])
        ref = O.verify_greedy_target_block(int(anchors[s]), c_s, D, vocab, t_s)
        assert st[s] == ref[0], (s, st[s], ref)
        if ref[0] == 0:
            assert acc[s] == ref[1] and np.array_equal(com[s, :acc[s] + 1], ref[2]), s
    assert st[3] == 9 and st[5] == 9 and st[7] == 9 and st[9] == 16
