"""Test fixture writer for K3X v1 containers holding MXFP4 expert records --
TEST INFRASTRUCTURE ONLY.

Restates the container layout of converter/k3x_converter/format.py (superblock
:80-104, tensor records :155-185, layer :199-213 and expert :222-236 records,
directories :258-263, root digest :296-315) for one MoE layer: per expert the
three MXFP4 projections `<prefix>.{gate,up,down}` as UINT8 records with an
E8M0 auxiliary extent, every extent 4096-aligned, CRC32C and SHA-256 digests
filled in. tests/test_k3x_reader.py checks that the reference's own C++ reader
accepts what this writes.
"""
from __future__ import annotations

import hashlib
import struct
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden" / "_shims"))
import google_crc32c  # noqa: E402  (pure-Python CRC-32C)

BLOCK = 4096


def fnv1a64(name: str) -> int:
    h = 0xCBF29CE484222325
    for byte in name.encode("utf-8"):
        h ^= byte
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _align(n: int) -> int:
    return (n + BLOCK - 1) // BLOCK * BLOCK


def write_mxfp4_experts(path: Path, experts: dict) -> None:
    """experts: {prefix: (expert_id or -1, {role: (packed u8 [r, c/2], scales u8 [r, c/32], (r, c))})}
    in layer 0."""
    records, payload = [], []
    expert_rows = []
    offset_cursor = [0]  # filled after the directories are sized
    items = []
    for prefix, (eid, roles) in experts.items():
        ids = {}
        for role in ("gate", "up", "down"):
            packed, scales, (rows, cols) = roles[role]
            tid = fnv1a64(f"{prefix}.{role}")
            ids[role] = tid
            items.append((tid, eid, packed.tobytes(), scales.tobytes(), rows, cols))
        if eid >= 0:
            expert_rows.append((eid, ids))
    n_t, n_e = len(items), len(expert_rows)
    tdir_len = 16 + 128 * n_t
    ldir_len = 16 + 64
    edir_len = 16 + 64 * n_e
    off = BLOCK
    tdir_off = off; off = _align(off + tdir_len)
    ldir_off = off; off = _align(off + ldir_len)
    edir_off = off; off = _align(off + edir_len)
    cfg_off = off; off = _align(off + 256)
    body = []
    for tid, eid, data, aux, rows, cols in items:
        d_off = off; off = _align(off + len(data))
        a_off = off; off = _align(off + len(aux))
        rec = bytearray(128)
        struct.pack_into("<QIHHBBHiiI", rec, 0, tid, 0, 2, 1, 2, 0, 0, 0, eid, 0)
        struct.pack_into("<4Q5QII", rec, 32, rows, cols, 0, 0, d_off, len(data), rows * cols,
                         a_off, len(aux), google_crc32c.value(data), google_crc32c.value(aux))
        records.append(bytes(rec))
        body.append((d_off, data))
        body.append((a_off, aux))
    file_len = off
    tdir = struct.pack("<4sIQ", b"TENS", 128, n_t) + b"".join(records)
    layer = bytearray(64)
    struct.pack_into("<IHHIIIIiI", layer, 0, 0, 1, 2, 0, n_t, 0, n_e, 0, 0)
    ldir = struct.pack("<4sIQ", b"LAYR", 64, 1) + bytes(layer)
    erecs = []
    for order, (eid, ids) in enumerate(expert_rows):
        r = bytearray(64)
        struct.pack_into("<IIIIQQQQ", r, 0, 0, eid, order, 0, ids["gate"], ids["up"], ids["down"], 0)
        erecs.append(bytes(r))
    edir = struct.pack("<4sIQ", b"EXPT", 64, n_e) + b"".join(erecs)
    cfg = bytearray(256)
    struct.pack_into("<I", cfg, 8, 1)  # layer count
    struct.pack_into("<I", cfg, 48, max([e for e, _ in expert_rows], default=0) + 1)
    image = bytearray(file_len)
    for o, blob in [(tdir_off, tdir), (ldir_off, ldir), (edir_off, edir), (cfg_off, bytes(cfg))] + body:
        image[o:o + len(blob)] = blob
    sb = bytearray(BLOCK)
    struct.pack_into("<8sHHIIIQQ", sb, 0, b"K3XCHKPT", 1, 0, BLOCK, BLOCK, 1, 0, 0)
    sb[40:56] = bytes(range(16))
    sb[56:88] = hashlib.sha256(b"test fixture").digest()
    struct.pack_into("<10Q", sb, 88, tdir_off, len(tdir), ldir_off, len(ldir), edir_off, len(edir),
                     cfg_off, 256, BLOCK, file_len)
    sb[168:200] = hashlib.sha256(tdir + ldir + edir + bytes(cfg)).digest()
    image[:BLOCK] = sb
    sb[200:232] = hashlib.sha256(bytes(image)).digest()  # root: digest and CRC fields zero
    struct.pack_into("<I", sb, 4092, google_crc32c.value(bytes(sb[:4092])))
    image[:BLOCK] = sb
    Path(path).write_bytes(bytes(image))
