"""Routing policy (natural / fixed / adaptive Top-K of select_routing) on CPU:
the oracle's C restatement (oracle/glm5x_oracle.c orc_select_routing_policy)
against the reference's own test expectations, against the reference's C++
compiled in oracle/_ref, and the C ABI's configuration checks (no GPU work).

Golden vectors: tests/cpp/test_routing_policy.cpp:31-133 and
tests/python/test_adaptive_routing_reference.py:46-80 of the reference.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle as O

SP = O.select_routing_policy


@pytest.mark.parametrize("use_reference", [False, True])
def test_reference_vectors(use_reference):
    if use_reference and O.ref_lib() is None:
        pytest.skip("oracle/_ref not built")
    kw = dict(use_reference=use_reference)
    # natural order with a bias, ties to the lower index (test_routing_policy.cpp:31-47)
    ids, w, k, esc, diag = SP([0.8, 0.8, 0.4, 0.7, 0.2, 0.1], [0, 0, 0.5, 0, 0, 0], 4, **kw)
    assert ids.tolist() == [2, 0, 1, 3] and k == 4 and not esc
    assert np.allclose(w, np.array([0.4, 0.8, 0.8, 0.7]) / 2.7, atol=1e-6)
    assert abs(diag[2] - 1.0) < 1e-6
    # natural mode ignores the floor (:48-53)
    _, _, k, esc, _ = SP([0.8, 0.8, 0.4, 0.7, 0.2, 0.1], [0, 0, 0.5, 0, 0, 0], 4,
                         quality_floor_k=16, **kw)
    assert k == 4 and not esc
    # fixed K = 4 of a natural Top-16 (:55-70)
    desc = [1.0 - i * 0.04 for i in range(16)]
    ids, w, k, _, diag = SP(desc, [0] * 16, 16, "fixed", fixed_k=4, **kw)
    assert k == 4 and ids[:4].tolist() == [0, 1, 2, 3] and (ids[4:] == -1).all()
    assert abs(w.sum() - 1.0) < 1e-6 and diag[2] < 1.0
    # adaptive: eight supported experts (:72-82)
    eight = [1.0] * 8 + [1e-9] * 8
    ids, w, k, _, diag = SP(eight, [0] * 16, 16, "adaptive", mass_target=0.75,
                            minimum_boundary_gap=0.1, **kw)
    assert k == 8 and ids[:8].tolist() == list(range(8))
    assert diag[1] <= 8.0001 and diag[3] > 0.9
    # quality floor escalation (:84-92)
    _, _, k, esc, _ = SP(eight, [0] * 16, 16, "adaptive", mass_target=0.75,
                         quality_floor_k=12, **kw)
    assert k == 12 and esc
    # weak boundary rejects every ladder K below 16 (:94-104)
    weak = [1.0] * 8 + [0.1] * 5 + [1e-9] * 3
    _, _, k, _, _ = SP(weak, [0] * 16, 16, "adaptive", mass_target=0.8,
                       minimum_boundary_gap=0.2, **kw)
    assert k == 16
    # invalid configurations and scores (:106-133)
    for args, kwargs in [((desc, [0] * 16, 16, "fixed"), dict(fixed_k=2)),
                         ((desc, [0] * 16, 12, "fixed"), dict(fixed_k=16)),
                         ((desc, [0] * 16, 16, "adaptive"), dict(mass_target=float("nan"))),
                         (([1.1] + desc[1:], [0] * 16, 16), {}),
                         (([0.0] * 16, [0] * 16, 16), {}),
                         ((desc, [0] * 16, 16, "adaptive"), dict(quality_floor_k=5)),
                         ((desc, [0] * 16, 8, "adaptive"), {})]:
        with pytest.raises(ValueError):
            SP(*args, **kwargs, **kw)


def _random_case(rng, n=256):
    scores = (1.0 / (1.0 + np.exp(-rng.normal(0, 2.0, n)))).astype(np.float32)
    if rng.random() < 0.3:  # peaked: a few dominant experts
        scores[rng.choice(n, 6, replace=False)] = rng.uniform(0.95, 1.0, 6).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    return scores, bias


def test_restatement_matches_reference_cpp():
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(5)
    configs = [("natural", dict(), 8), ("natural", dict(), 16), ("fixed", dict(fixed_k=4), 8),
               ("fixed", dict(fixed_k=6, quality_floor_k=8), 16),
               ("adaptive", dict(mass_target=0.9), 16),
               ("adaptive", dict(mass_target=0.6, minimum_boundary_gap=0.05), 16),
               ("adaptive", dict(mass_target=0.5, quality_floor_k=8), 16)]
    for _ in range(300):
        s, b = _random_case(rng)
        for mode, kw, k in configs:
            a = SP(s, b, k, mode, **kw)
            r = SP(s, b, k, mode, **kw, use_reference=True)
            assert np.array_equal(a[0], r[0]) and np.array_equal(a[1], r[1])
            assert a[2:4] == r[2:4]
            assert np.array_equal(a[4], r[4])


def test_c_abi_rejects_invalid_policies_before_device_work():
    """The library's checks mirror select_routing's messages; every call here
    fails validation, so no device memory is touched."""
    from glm5x_moe import _native as N
    from glm5x_moe.routing import RoutingMode, RoutingPolicyConfig
    lib = N.lib()
    dummy = ctypes.c_void_p(16)
    cases = [(RoutingPolicyConfig(RoutingMode.FIXED, fixed_k=2), 16, b"invalid fixed routing K"),
             (RoutingPolicyConfig(RoutingMode.FIXED, fixed_k=16), 12, b"invalid fixed routing K"),
             (RoutingPolicyConfig(RoutingMode.ADAPTIVE), 8,
              b"adaptive routing requires natural Top-16"),
             (RoutingPolicyConfig(RoutingMode.ADAPTIVE, mass_target=float("nan")), 16,
              b"invalid adaptive routing threshold"),
             (RoutingPolicyConfig(RoutingMode.ADAPTIVE, minimum_boundary_gap=1.5), 16,
              b"invalid adaptive routing threshold"),
             (RoutingPolicyConfig(RoutingMode.ADAPTIVE, quality_floor_k=5), 16,
              b"invalid routing quality floor")]
    for cfg, k, msg in cases:
        pol = cfg.to_c()
        rc = lib.glm5x_select_routing_policy(dummy, dummy, 4, 256, k, ctypes.byref(pol), 1.0,
                                             dummy, dummy, None, None, None)
        assert rc == 16, (cfg, rc)
        assert msg in lib.glm5x_last_error_message(), lib.glm5x_last_error_message()
