"""K3X v1 containers through the C ABI (no GPU): the container written by the
reference's own converter (tests/golden/make_k3x_golden.py) opens with every
checksum verified, its records read back byte for byte as the reference's C++
reader (oracle/_ref) reads them, every corruption is rejected with the status
that reader returns, and the test-side writer of GLM-shaped MXFP4 experts
(tests/k3x_fixture.py) produces files the reference's reader accepts.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from k3x_fixture import write_mxfp4_experts

GOLDEN = Path(__file__).resolve().parent / "golden" / "k3x_small.k3x"
# MoE layers 1-3 of the synthetic K3 model, two experts each, plus dense tensors
EXPERT_NAMES = [f"model.layers.{l}.feed_forward.experts.{e}.{r}"
                for l in (1, 2, 3) for e in (0, 1) for r in ("gate", "up", "down")]
PLAIN_NAMES = ["model.layers.1.attention.q_proj", "model.layers.1.feed_forward.correction_bias"]


def _status(fn):
    from glm5x_moe._native import Glm5xError
    try:
        fn()
    except Glm5xError as e:
        return e.code
    return 0


def test_reference_container_reads_back():
    from glm5x_moe.k3x import K3xFile, fnv1a64
    with K3xFile(GOLDEN, verify=True) as f:
        for name in EXPERT_NAMES + PLAIN_NAMES:
            rec = f.tensor(name)
            data, aux = f.read(name)
            assert rec["tensor_id"] == fnv1a64(name)
            if name in EXPERT_NAMES:
                assert rec["dtype"] == 2 and rec["quantization"] == 1 and rec["rank"] == 2
                r, c = rec["shape"]
                assert data.size == r * c // 2 and aux.size == r * c // 32
            else:
                assert rec["quantization"] == 0 and aux is None
            if O.ref_lib() is not None:
                rc, rd, ra = O.ref_k3x_read(GOLDEN, fnv1a64(name))
                assert rc == 0 and np.array_equal(rd, data)
                assert np.array_equal(ra, aux if aux is not None else np.zeros(0, np.uint8))
        assert _status(lambda: f.tensor("model.layers.9.absent")) == 14


def _variants(tmp_path):
    good = GOLDEN.read_bytes()
    import sys
    sys.path.insert(0, str(GOLDEN.parent / "_shims"))
    import google_crc32c

    def with_crc(b):
        b = bytearray(b)
        struct.pack_into("<I", b, 4092, google_crc32c.value(bytes(b[:4092])))
        return bytes(b)

    def flip(b, i):
        b = bytearray(b)
        b[i] ^= 1
        return bytes(b)

    required = bytearray(good)
    struct.pack_into("<Q", required, 24, 1)
    version = bytearray(good)
    struct.pack_into("<H", version, 8, 2)
    tdir_off = struct.unpack_from("<Q", good, 88)[0]
    first_data = struct.unpack_from("<Q", good, tdir_off + 16 + 64)[0]  # first record's data
    out = {"magic": b"K3XCHKPX" + good[8:], "version": with_crc(version),
           "superblock_crc": flip(good, 300), "required": with_crc(required),
           "truncated": good[:-4096], "short": good[:1000], "payload": flip(good, first_data + 5)}
    st = bytearray(good)
    struct.pack_into("<I", st, 20, 0)
    out["state"] = with_crc(st)
    rec_reserved = bytearray(good)
    rec_reserved[tdir_off + 16 + 120] = 1  # reserved bytes of the first tensor record
    out["record"] = bytes(rec_reserved)
    paths = {}
    for k, v in out.items():
        p = tmp_path / f"{k}.k3x"
        p.write_bytes(v)
        paths[k] = p
    return paths


def test_rejections_match_reference_reader(tmp_path):
    from glm5x_moe.k3x import K3xFile
    expect = {"magic": 2, "version": 3, "superblock_crc": 6, "required": 4, "truncated": 7,
              "short": 7, "state": 7}
    paths = _variants(tmp_path)
    for k, code in expect.items():
        for verify in (False, True):
            assert _status(lambda: K3xFile(paths[k], verify=verify)) == code, (k, verify)
            if O.ref_lib() is not None:
                assert O.ref_k3x_open(paths[k], verify) == code, (k, verify)
    # a flipped payload byte passes the metadata checks and fails the digests
    assert _status(lambda: K3xFile(paths["payload"], verify=False)) == 0
    got = _status(lambda: K3xFile(paths["payload"], verify=True))
    assert got in (10, 11, 13)
    # a directory byte changed after the digest: the metadata checks reject the record
    assert _status(lambda: K3xFile(paths["record"], verify=False)) == 8
    if O.ref_lib() is not None:
        assert O.ref_k3x_open(paths["payload"], True) == got
        assert O.ref_k3x_open(paths["payload"], False) == 0
        assert O.ref_k3x_open(paths["record"], False) == 8


def test_fixture_writer_accepted_by_reference_reader(tmp_path):
    from glm5x_moe.k3x import K3xFile
    rng = np.random.default_rng(3)

    def mat(r, c):
        return (rng.integers(0, 256, (r, c // 2), dtype=np.uint8),
                rng.integers(110, 130, (r, c // 32), dtype=np.uint8), (r, c))

    experts = {f"model.layers.0.feed_forward.experts.{e}": (e, {
        "gate": mat(512, 512), "up": mat(512, 512), "down": mat(512, 512)}) for e in range(2)}
    experts["model.layers.0.feed_forward.shared_experts.0"] = (-1, {
        "gate": mat(512, 512), "up": mat(512, 512), "down": mat(512, 512)})
    p = tmp_path / "fixture.k3x"
    write_mxfp4_experts(p, experts)
    with K3xFile(p, verify=True) as f:
        for prefix, (_, roles) in experts.items():
            for role, (packed, scales, shape) in roles.items():
                data, aux = f.read(f"{prefix}.{role}")
                assert np.array_equal(data, packed.reshape(-1))
                assert np.array_equal(aux, scales.reshape(-1))
    if O.ref_lib() is not None:
        assert O.ref_k3x_open(p, True) == 0
