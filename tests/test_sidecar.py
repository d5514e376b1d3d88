"""Packed expert sidecars (.pn4 / .pm4) on the CPU: the library's reader
(glm5x_sidecar_open, the host half of glm5x_moe_load_sidecar) against files
written by the reference's own GLM5XPackedExpertCache.put
(tests/golden/make_sidecar_golden.py) and against every check of the
reference's get / _decode_role (packed_cache.py:506-545, 407-479), in its
order. No GPU is used.
"""
from __future__ import annotations

import hashlib
import json
import struct
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from sidecar_fixture import crc32c, mxfp4_role, nvfp4_role, sidecar_bytes

REPO = Path(__file__).resolve().parents[1]
GOLD = REPO / "tests" / "golden" / "sidecar"
EXPECTED = json.loads((GOLD / "expected.json").read_text())
DIGEST = EXPECTED["source_digest"]
NV = GOLD / "layer-0010-expert-0003.pn4"
MX = GOLD / "layer-0010-expert-0004.pm4"


def _sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def test_crc32c_check_value():
    assert crc32c(b"123456789") == 0xE3069283


def test_reads_reference_nvfp4_sidecar():
    from glm5x_moe.sidecar import read_sidecar
    roles = read_sidecar(NV, "nvfp4", DIGEST)
    want = EXPECTED["files"][NV.name]["roles"]
    for got, exp in zip(roles, want):
        assert got.precision == "nvfp4" and list(got.shape) == exp["shape"]
        assert _sha(got.packed) == exp["packed_sha256"]
        assert _sha(got.scales) == exp["scales_sha256"]
        assert np.float32(got.global_scale) == np.float32(exp["global_scale"])


def test_reads_reference_mxfp4_sidecar():
    """The MXFP4 bytes the reader returns decode (oracle decode_mxfp4) to the
    BF16 weights the reference's own reader decodes from the same file."""
    from glm5x_moe.sidecar import read_sidecar
    roles = read_sidecar(MX, "mxfp4", DIGEST)
    want = EXPECTED["files"][MX.name]["roles"]
    for got, exp in zip(roles, want):
        assert got.precision == "mxfp4" and list(got.shape) == exp["shape"]
        rows, cols = got.shape
        dec = O.mxfp4_decode(np.frombuffer(got.packed, np.uint8),
                             np.frombuffer(got.scales, np.uint8), rows, cols)
        bf16 = (O.bf16_round(dec).view(np.uint32) >> 16).astype(np.uint16)
        assert _sha(bf16.tobytes()) == exp["decoded_bf16_sha256"]


def test_writer_reproduces_reference_files():
    """The test-side writer (used for GLM-layout sidecars on the GPU) gives
    the reference's bytes back from the roles the reader returns."""
    from glm5x_moe.sidecar import read_sidecar
    nv = read_sidecar(NV)
    assert sidecar_bytes("nvfp4", DIGEST, [nvfp4_role(r.packed, r.scales, r.global_scale, r.shape)
                                           for r in nv]) == NV.read_bytes()
    mx = read_sidecar(MX)
    assert sidecar_bytes("mxfp4", DIGEST, [mxfp4_role(r.packed, r.scales, r.shape)
                                           for r in mx]) == MX.read_bytes()


def test_sidecar_path_matches_reference_naming():
    from glm5x_moe.sidecar import sidecar_path
    assert sidecar_path("/x", (10, 3), "nvfp4") == Path("/x/layer-0010-expert-0003.pn4")
    assert sidecar_path("/x", (0, 255), "mxfp4") == Path("/x/layer-0000-expert-0255.pm4")
    from glm5x_moe._native import Glm5xError
    with pytest.raises(Glm5xError, match="GLM5X_PACKED_CACHE_KEY"):
        sidecar_path("/x", (-1, 0), "nvfp4")


def _split(data: bytes):
    _, _, mlen = struct.unpack_from("<8sII", data)
    return json.loads(data[16:16 + mlen]), bytearray(data[16 + mlen:])


def _join(meta: dict, payload: bytes, version: int = 1, magic: bytes = b"GLM5XPI4") -> bytes:
    enc = json.dumps(meta, sort_keys=True, separators=(",", ":")).encode()
    return struct.pack("<8sII", magic, version, len(enc)) + enc + bytes(payload)


def _corrupt(name: str, data: bytes) -> bytes:
    meta, payload = _split(data)
    r0 = meta["roles"][0]
    if name == "header":
        return data[:12]
    if name == "magic":
        return _join(meta, payload, magic=b"GLM5XPI5")
    if name == "version":
        return _join(meta, payload, version=2)
    if name == "metadata":
        return data[:16] + b"[" + data[17:]
    if name == "format":
        meta["format"] = "glm5x-int4-expert-v1"
    elif name == "digest":
        meta["source_digest"] = "0" * 32
    elif name == "roles":
        meta["roles"] = meta["roles"][:2]
    elif name == "payload":
        payload += b"\0"
    elif name == "extent":
        r0["packed_bytes"] = len(payload) + 1
    elif name == "packed_crc":
        payload[r0["packed_offset"]] ^= 1
    elif name == "qparam_crc":
        payload[r0["qparams_offset"]] ^= 1
    elif name == "nvfp4_qparam":
        r0["scale_bytes"] -= 4
    elif name == "crc_before_qparam_extent":
        # two faults: the reference meets the CRC first
        payload[r0["packed_offset"]] ^= 1
        r0["scale_bytes"] -= 4
    return _join(meta, payload)


CASES = [("header", 7, "HEADER"), ("magic", 2, "FORMAT"), ("version", 3, "FORMAT"),
         ("metadata", 8, "METADATA"), ("format", 16, "FORMAT"),
         ("digest", 16, "SOURCE_MISMATCH"), ("roles", 8, "ROLES"),
         ("payload", 9, "PAYLOAD_EXTENT"), ("extent", 9, "PAYLOAD_EXTENT"),
         ("packed_crc", 10, "PACKED_CRC"), ("qparam_crc", 11, "QPARAM_CRC"),
         ("nvfp4_qparam", 9, "NVFP4_QPARAM_EXTENT"),
         ("crc_before_qparam_extent", 10, "PACKED_CRC")]


@pytest.mark.parametrize("name,status,code", CASES)
def test_rejects_what_the_reference_rejects(tmp_path, name, status, code):
    from glm5x_moe._native import Glm5xError
    from glm5x_moe.sidecar import read_sidecar
    p = tmp_path / NV.name
    p.write_bytes(_corrupt(name, NV.read_bytes()))
    with pytest.raises(Glm5xError) as ei:
        read_sidecar(p, "nvfp4", DIGEST)
    assert ei.value.code == status, (name, ei.value)
    assert f"GLM5X_PACKED_CACHE_{code}" in str(ei.value), (name, ei.value)


def test_precision_and_digest_are_optional_filters(tmp_path):
    from glm5x_moe._native import Glm5xError
    from glm5x_moe.sidecar import read_sidecar
    assert read_sidecar(NV)[0].precision == "nvfp4"  # the file's own format
    with pytest.raises(Glm5xError, match="GLM5X_PACKED_CACHE_FORMAT"):
        read_sidecar(NV, "mxfp4")
    with pytest.raises(Glm5xError, match="GLM5X_PACKED_CACHE_IO"):
        read_sidecar(tmp_path / "absent.pn4")
