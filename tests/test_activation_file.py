"""GLM5XACT activation files through the C ABI (no GPU): the fixture written
by the reference's own writer (tests/golden/make_activation_golden.py) reads
back to the values it was written from, this build's writer reproduces it
byte for byte, and every rejection of the reference's reader
(runtime/src/glm5x_activation.cpp:53-109) maps to the same status.
"""
from __future__ import annotations

import struct
import sys
from pathlib import Path

import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))

from make_activation_golden import pattern  # noqa: E402


def test_reads_reference_fixture_and_writes_identical_bytes(tmp_path):
    from glm5x_moe.activation import load_bf16_activation, write_bf16_activation
    src = GOLDEN / "activation_small.glm5xact"
    x = load_bf16_activation(src, expected_token_count=5, expected_hidden_size=48)
    assert x.dtype == torch.bfloat16 and tuple(x.shape) == (5, 48)
    assert torch.equal(x.view(torch.int16), pattern(5, 48).view(torch.int16))
    out = tmp_path / "sub" / "copy.glm5xact"
    write_bf16_activation(out, x.float())
    assert out.read_bytes() == src.read_bytes()


def _status(fn):
    from glm5x_moe._native import Glm5xError
    with pytest.raises(Glm5xError) as e:
        fn()
    return e.value.name


def test_rejections_match_reference_reader(tmp_path):
    from glm5x_moe.activation import load_bf16_activation
    good = (GOLDEN / "activation_small.glm5xact").read_bytes()

    def variant(name, data):
        p = tmp_path / name
        p.write_bytes(data)
        return lambda: load_bf16_activation(p)

    hdr = bytearray(good[:40])
    assert _status(lambda: load_bf16_activation(tmp_path / "absent")) == "IO_ERROR"
    assert _status(variant("short", good[:30])) == "TRUNCATED_FILE"
    assert _status(variant("magic", b"GLM5XACX" + good[8:])) == "BAD_MAGIC"
    for off, val, fmt in [(8, 2, "<I"), (12, 41, "<I"), (24, 1, "<H"), (26, 1, "<H")]:
        h = bytearray(hdr)
        struct.pack_into(fmt, h, off, val)
        assert _status(variant(f"v{off}", bytes(h) + good[40:])) == "UNSUPPORTED_VERSION", off
    h = bytearray(hdr)
    struct.pack_into("<I", h, 16, 0)
    assert _status(variant("zero", bytes(h) + good[40:])) == "INVALID_EXTENT"
    assert _status(variant("long", good + b"\0\0")) == "INVALID_EXTENT"
    assert _status(lambda: load_bf16_activation(GOLDEN / "activation_small.glm5xact",
                                                expected_token_count=4)) == "INVALID_EXTENT"
    assert _status(lambda: load_bf16_activation(GOLDEN / "activation_small.glm5xact",
                                                expected_hidden_size=64)) == "INVALID_EXTENT"
    flipped = bytearray(good)
    flipped[100] ^= 1
    assert _status(variant("crc", bytes(flipped))) == "DATA_CRC_MISMATCH"


def test_writer_rejects_empty_and_rank(tmp_path):
    from glm5x_moe.activation import write_bf16_activation
    with pytest.raises(ValueError):
        write_bf16_activation(tmp_path / "a", torch.zeros(3))
    with pytest.raises(ValueError):
        write_bf16_activation(tmp_path / "b", torch.zeros(0, 4))
