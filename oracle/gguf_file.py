"""GGUF header reader restated in plain Python (test infrastructure: the checker for the library's
native reader, never on the product path).

Follows candle-core's quantized/gguf_file.rs (vendor/candle-core/src/quantized/gguf_file.rs):
  28-33    length prefixes: u32 in version 1, u64 in versions 2 and 3
  40-70    magic 0x46554747 or 0x47475546 read as a little-endian u32, versions 1..3
  130-150  strings: length, bytes, trailing NULs dropped, decoded leniently
  319-375  metadata values by type id (arrays typed, nested arrays allowed to depth 64)
  469-563  Content::read: counts checked against the file's size, metadata, tensor infos
           (dims innermost first on disk, at most 4; u32 dims in version 1), alignment from
           general.alignment when it is an 8/16/32-bit integer (signed ones when >= 0) else 32,
           tensor data at the header's end rounded up to that alignment.
"""

from __future__ import annotations

import struct

MAX_COUNT = 1 << 30
MAX_DEPTH = 64
_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q", 11: "<q", 12: "<d"}
STRING, ARRAY, BOOL = 8, 9, 7


class GgufError(ValueError):
    pass


class _Reader:
    def __init__(self, data: bytes):
        self.d, self.p, self.v1 = data, 0, False

    def take(self, fmt: str):
        n = struct.calcsize(fmt)
        if self.p + n > len(self.d):
            raise GgufError("truncated")
        v = struct.unpack_from(fmt, self.d, self.p)[0]
        self.p += n
        return v

    def length(self) -> int:
        return self.take("<I" if self.v1 else "<Q")

    def string(self) -> str:
        n = self.length()
        if n > MAX_COUNT or n > len(self.d) - self.p:
            raise GgufError("string longer than the file")
        b = self.d[self.p:self.p + n].rstrip(b"\0")
        self.p += n
        return b.decode("utf-8", errors="replace")

    def value(self, t: int, depth: int = 0):
        if depth > MAX_DEPTH:
            raise GgufError("metadata nested too deep")
        if t in _SCALARS:
            v = self.take(_SCALARS[t])
            if t == BOOL and v > 1:
                raise GgufError("bool value other than 0 or 1")
            return bool(v) if t == BOOL else v
        if t == STRING:
            return self.string()
        if t == ARRAY:
            et = self.take("<I")
            n = self.length()
            if n > MAX_COUNT:
                raise GgufError("array too long")
            return [self.value(et, depth + 1) for _ in range(n)]
        raise GgufError(f"unknown metadata value type {t}")


def read(data: bytes) -> dict:
    """{version, metadata {key: (type, value)}, tensors {name: (ne innermost first, ggml type,
    offset)}, alignment, data_offset}."""
    r = _Reader(data)
    magic = r.take("<I")
    if magic not in (0x46554747, 0x47475546):
        raise GgufError("bad magic")
    version = r.take("<I")
    if version not in (1, 2, 3):
        raise GgufError("unsupported version")
    r.v1 = version == 1
    n_tensors, n_kv = r.length(), r.length()
    pre = 4 if r.v1 else 8
    if n_tensors > MAX_COUNT or n_kv > MAX_COUNT or n_kv * (pre + 5) + n_tensors * (pre + 16) > len(data) - r.p:
        raise GgufError("header counts out of range")
    meta = {}
    for _ in range(n_kv):
        key = r.string()
        t = r.take("<I")
        meta[key] = (t, r.value(t))
    tensors = {}
    for _ in range(n_tensors):
        name = r.string()
        nd = r.take("<I")
        if nd > 4:
            raise GgufError("more than 4 dimensions")
        ne = [r.take("<I" if r.v1 else "<Q") for _ in range(nd)]
        tensors[name] = (ne, r.take("<I"), r.take("<Q"))
    alignment = 32
    if "general.alignment" in meta:
        t, v = meta["general.alignment"]
        if t in (0, 2, 4) or (t in (1, 3, 5) and v >= 0):
            alignment = v
    if alignment == 0:
        raise GgufError("general.alignment is 0")
    data_offset = (r.p + alignment - 1) // alignment * alignment
    return dict(version=version, metadata=meta, tensors=tensors, alignment=alignment, data_offset=data_offset)
