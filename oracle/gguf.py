"""CPU restatement of the engine's GGUF v3 parse (test infrastructure only).

Follows ds3_gguf_open, src/ds3_gguf.c:179-356 of wzqhbustb/qw3: header
(:214-236), metadata pairs with the general.alignment override (:238-262),
tensor infos (:264-290), data region at the next multiple of the alignment
(:292-296), per-tensor data pointer and size from the block table, a partial
trailing block counted whole (:298-344). Byte strides follow make_tensor,
src/ds3_weights.c:63-95. Only tests import this module.
"""

from __future__ import annotations

import struct

_SCALAR = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
GEOMETRY = {0: (4, 1), 1: (2, 1), 2: (18, 32), 6: (22, 32), 8: (34, 32), 10: (84, 256), 11: (110, 256),
            12: (144, 256), 13: (176, 256), 14: (210, 256), 15: (290, 256), 16: (66, 256), 17: (74, 256),
            18: (98, 256)}


class ParseError(ValueError):
    pass


class _Cur:
    def __init__(self, b: bytes):
        self.b, self.p = b, 0

    def take(self, n: int) -> bytes:
        if n < 0 or self.p + n > len(self.b):
            raise ParseError("read past end of file")
        out = self.b[self.p:self.p + n]
        self.p += n
        return out

    def u32(self) -> int:
        return struct.unpack("<I", self.take(4))[0]

    def u64(self) -> int:
        return struct.unpack("<Q", self.take(8))[0]

    def string(self) -> bytes:
        return self.take(self.u64())


def _value(c: _Cur, t: int):
    if t in _SCALAR:
        raw = c.take(_SCALAR[t])
        fmt = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q",
               12: "<d"}[t]
        return struct.unpack(fmt, raw)[0]
    if t == 8:
        return c.string()
    if t == 9:
        et, n = c.u32(), c.u64()
        return [_value(c, et) for _ in range(n)]
    raise ParseError(f"unknown metadata value type {t}")


def parse(data: bytes) -> dict:
    """Header fields, metadata {key: (type, value)} and the tensor table."""
    c = _Cur(data)
    if c.take(4) != b"GGUF":
        raise ParseError("bad magic")
    version = c.u32()
    if version < 3:
        raise ParseError("version < 3")
    n_tensors, n_meta = c.u64(), c.u64()
    meta, alignment = {}, 32
    for _ in range(n_meta):
        key = c.string().decode("utf-8", "replace")
        t = c.u32()
        v = _value(c, t)
        meta.setdefault(key, (t, v))
        if key == "general.alignment" and t == 4:
            alignment = v
    if alignment == 0:
        raise ParseError("alignment 0")
    infos = []
    for _ in range(n_tensors):
        name = c.string().decode("utf-8", "replace")
        n_dims = c.u32()
        if n_dims > 4:
            raise ParseError("more than 4 dimensions")
        ne = [c.u64() for _ in range(n_dims)]
        t, off = c.u32(), c.u64()
        infos.append((name, n_dims, ne, t, off))
    data_offset = c.p + (alignment - c.p % alignment) % alignment
    table = []
    for name, n_dims, ne, t, off in infos:
        if t not in GEOMETRY:
            raise ParseError(f"unknown tensor type {t}")
        bb, be = GEOMETRY[t]
        n = 1
        for x in ne:
            n *= x
        size = (n // be) * bb + (bb if n % be else 0)
        ne4 = ne + [1] * (4 - n_dims)
        nb = [bb if n_dims else 0, bb * (ne4[0] // be) if n_dims >= 2 else 0, 0, 0]
        for d in (2, 3):
            nb[d] = nb[d - 1] * ne4[d - 1]
        if data_offset + off + size > len(data):
            raise ParseError(f"tensor {name} runs past the end of the file")
        table.append({"name": name, "n_dims": n_dims, "ne": ne4, "nb": nb, "type": t, "offset": off,
                      "size": size})
    return {"version": version, "alignment": alignment, "data_offset": data_offset, "n_metadata": n_meta,
            "meta": meta, "tensors": table}
