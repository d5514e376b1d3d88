"""Test-side writer of packed expert sidecars in the layout of the
reference's GLM5XPackedExpertCache.put (reference/glm5x_ref/packed_cache.py:
224-327 records, 327-404 file): header "<8sII", compact sorted-key JSON,
payload of packed bytes then qparams per role. tests/test_sidecar.py pins it
by rewriting the reference-written fixtures under tests/golden/sidecar byte
for byte; the GPU tests use it for GLM-layout experts."""
from __future__ import annotations

import json
import struct
from pathlib import Path


def crc32c(data: bytes) -> int:
    """CRC-32C (Castagnoli, reflected 0x82F63B78), the google_crc32c value."""
    crc = 0xFFFFFFFF
    table = _table()
    for b in data:
        crc = table[(crc ^ b) & 0xFF] ^ (crc >> 8)
    return crc ^ 0xFFFFFFFF


_TAB: list[int] = []


def _table() -> list[int]:
    if not _TAB:
        for i in range(256):
            c = i
            for _ in range(8):
                c = (c >> 1) ^ 0x82F63B78 if c & 1 else c >> 1
            _TAB.append(c)
    return _TAB


def nvfp4_role(packed: bytes, scales: bytes, global_scale: float, shape) -> dict:
    """(record, packed, qparams) of one NVFP4 projection (_weight_payload's
    nvfp4 branch): qparams = blocked E4M3 scale bytes + FP32 global."""
    qparams = scales + struct.pack("<f", global_scale)
    rows, cols = shape
    rec = {"representation": "nvfp4", "shape": [rows, cols], "group_size": 16,
           "inner_k_tiles": 0, "packed_shape": [rows, cols // 2],
           "qparams_shape": [len(scales)], "qparams_dtype": "float8_e4m3fn",
           "packed_bytes": len(packed), "qparams_bytes": len(qparams),
           "scale_bytes": len(scales), "global_scale_bytes": 4,
           "packed_crc32c": crc32c(packed), "qparams_crc32c": crc32c(qparams)}
    return {"record": rec, "packed": packed, "qparams": qparams}


def mxfp4_role(packed: bytes, scales: bytes, shape) -> dict:
    """(record, packed, qparams) of one MXFP4 projection (_weight_payload's
    mxfp4 branch: encode_mxfp4 bytes, group 32, row-major E8M0)."""
    rows, cols = shape
    rec = {"shape": [rows, cols], "group_size": 32, "inner_k_tiles": 0,
           "packed_shape": [len(packed)], "qparams_shape": [len(scales)],
           "qparams_dtype": "uint8", "packed_bytes": len(packed), "qparams_bytes": len(scales),
           "packed_crc32c": crc32c(packed), "qparams_crc32c": crc32c(scales)}
    return {"record": rec, "packed": packed, "qparams": scales}


def sidecar_bytes(precision: str, source_digest: str, roles: list[dict]) -> bytes:
    records, payload = [], bytearray()
    for role in roles:
        rec = dict(role["record"])
        rec["packed_offset"] = len(payload)
        payload.extend(role["packed"])
        rec["qparams_offset"] = len(payload)
        payload.extend(role["qparams"])
        records.append(rec)
    meta = {"format": f"glm5x-{precision}-expert-v1", "source_digest": source_digest,
            "roles": records, "payload_bytes": len(payload)}
    enc = json.dumps(meta, sort_keys=True, separators=(",", ":")).encode("utf-8")
    return struct.pack("<8sII", b"GLM5XPI4", 1, len(enc)) + enc + bytes(payload)


def write_sidecar(path: Path, precision: str, source_digest: str, roles: list[dict]) -> None:
    Path(path).write_bytes(sidecar_bytes(precision, source_digest, roles))
