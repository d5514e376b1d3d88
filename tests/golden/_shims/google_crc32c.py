"""Pure-Python CRC-32C (Castagnoli) stand-in for the ``google_crc32c`` package.

Only the fixture generator imports this, so that the reference's Python modules
(which import ``google_crc32c`` at module load) can run in an environment where
the wheel is absent. Polynomial 0x82F63B78 (reflected), init/xorout 0xFFFFFFFF.
"""
from __future__ import annotations

_TABLE = []
for _i in range(256):
    _c = _i
    for _ in range(8):
        _c = (_c >> 1) ^ 0x82F63B78 if _c & 1 else _c >> 1
    _TABLE.append(_c)


def _update(crc: int, data: bytes) -> int:
    crc ^= 0xFFFFFFFF
    for b in data:
        crc = _TABLE[(crc ^ b) & 0xFF] ^ (crc >> 8)
    return crc ^ 0xFFFFFFFF


def value(data: bytes) -> int:
    return _update(0, bytes(data))


class Checksum:
    def __init__(self, initial_value: bytes = b"") -> None:
        self._crc = _update(0, bytes(initial_value))

    def update(self, data: bytes) -> None:
        self._crc = _update(self._crc, bytes(data))

    def digest(self) -> bytes:
        return self._crc.to_bytes(4, "big")

    def hexdigest(self) -> bytes:
        return self.digest().hex().encode()
