"""Greedy verification of speculative draft blocks on CPU: the oracle
restatement (orc_verify_greedy_target_block) against the reference's test
expectations (tests/cpp/test_speculative.cpp:155-240) and against the
reference's own C++ (oracle/_ref) on random blocks."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O

# (anchor, candidates, max_draft, vocab, targets) -> (status, accepted, committed)
CASES = [
    ((10, [11, 12], 2, 128, [11, 12, 13]), (0, 2, [11, 12, 13])),
    ((10, [99, 100], 2, 128, [11, 12, 13]), (0, 0, [11])),
    ((10, [11, 99], 2, 128, [11, 12, 13]), (0, 1, [11, 12])),
    ((10, [11, 12, 99], 3, 128, [11, 12, 13, 14]), (0, 2, [11, 12, 13])),
    ((10, [], 0, 128, [11]), (0, 0, [11])),
    ((10, [11, 12], 2, 128, [11, 12]), (9, 0, None)),
    ((10, [11, 12], 2, 128, [11, 12, 13, 14]), (9, 0, None)),
    ((10, [128], 1, 128, [11, 12]), (9, 0, None)),
    ((10, [11], 1, 128, [11, 128]), (16, 0, None)),
]


@pytest.mark.parametrize("use_reference", [False, True])
def test_reference_vectors(use_reference):
    if use_reference and O.ref_lib() is None:
        pytest.skip("oracle/_ref not built")
    for (anchor, cand, mx, vocab, tgt), (st, acc, com) in CASES:
        got = O.verify_greedy_target_block(anchor, cand, mx, vocab, tgt, use_reference)
        assert got[0] == st and got[1] == acc, (anchor, cand, tgt, got)
        if com is not None:
            assert got[2].tolist() == com


def test_restatement_matches_reference_cpp():
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(1)
    for _ in range(3000):
        vocab = int(rng.integers(2, 40))
        mx = int(rng.integers(0, 6))
        n = int(rng.integers(0, mx + 2))
        anchor = int(rng.integers(0, vocab + 1))
        cand = rng.integers(0, vocab + (1 if rng.random() < 0.05 else 0), n)
        tgt = cand.copy() if rng.random() < 0.5 else rng.integers(0, vocab, n)
        tgt = np.concatenate([tgt, rng.integers(0, vocab + (1 if rng.random() < 0.05 else 0), 1)])
        if rng.random() < 0.5 and n:
            k = int(rng.integers(0, n))
            tgt[k] = (cand[k] + 1) % vocab
        if rng.random() < 0.05:
            tgt = tgt[:-1]
        a = O.verify_greedy_target_block(anchor, cand, mx, vocab, tgt)
        r = O.verify_greedy_target_block(anchor, cand, mx, vocab, tgt, use_reference=True)
        assert a[0] == r[0] and a[1] == r[1], (anchor, cand, mx, vocab, tgt, a, r)
        if a[0] == 0:
            assert np.array_equal(a[2], r[2])
