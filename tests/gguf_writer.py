"""Minimal GGUF v3 writer for tests (test infrastructure).

Writes files in the layout the GGUF specification defines and the engine's
reader (src/ds3_gguf.c of wzqhbustb/qw3) parses: magic "GGUF", version,
tensor count, metadata count, metadata key/value pairs, tensor infos, padding
to the alignment, then tensor data with every tensor's offset a multiple of
the alignment. The synthetic model files hold the tensor names the engine
binds (src/ds3_weights.c:122-138) with seeded random contents, so loading a
real checkpoint can be exercised without one.
"""

from __future__ import annotations

import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

# metadata value types (GGUF specification)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
           U64: "<Q", I64: "<q", F64: "<d"}

# tensor types: (bytes per block, elements per block), src/ds3_gguf.c:314-330
GEOMETRY = {0: (4, 1), 1: (2, 1), 2: (18, 32), 6: (22, 32), 8: (34, 32), 10: (84, 256), 11: (110, 256),
            12: (144, 256), 13: (176, 256), 14: (210, 256), 15: (290, 256), 16: (66, 256), 17: (74, 256),
            18: (98, 256)}


def tensor_bytes(type_: int, ne) -> int:
    bb, be = GEOMETRY[type_]
    n = int(np.prod(ne, dtype=np.int64)) if len(ne) else 1
    return (n // be) * bb + (bb if n % be else 0)


def _str(s: bytes | str) -> bytes:
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def _value(t: int, v) -> bytes:
    if t in _SCALAR:
        return struct.pack(_SCALAR[t], v)
    if t == STRING:
        return _str(v)
    if t == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    raise ValueError(t)


@dataclass
class GgufFile:
    alignment: int | None = None        # written as general.alignment (uint32) when set
    version: int = 3
    magic: bytes = b"GGUF"
    meta: list = field(default_factory=list)      # (key, type, value)
    tensors: list = field(default_factory=list)   # (name, ne, type, raw bytes)

    def add_meta(self, key: str, t: int, v) -> None:
        self.meta.append((key, t, v))

    def add_tensor(self, name: str, ne, type_: int, data: bytes) -> None:
        assert len(data) == tensor_bytes(type_, ne), (name, len(data), tensor_bytes(type_, ne))
        self.tensors.append((name, list(ne), type_, bytes(data)))

    def layout(self) -> tuple[bytes, list[int], int]:
        """(header bytes up to the end of the tensor infos, offsets, data offset)."""
        align = self.alignment or 32
        meta = list(self.meta)
        if self.alignment is not None:
            meta = [("general.alignment", U32, self.alignment)] + meta
        offsets, off = [], 0
        for _, ne, t, data in self.tensors:
            off = (off + align - 1) // align * align
            offsets.append(off)
            off += len(data)
        h = self.magic + struct.pack("<IQQ", self.version, len(self.tensors), len(meta))
        for k, t, v in meta:
            h += _str(k) + struct.pack("<I", t) + _value(t, v)
        for (name, ne, t, _), o in zip(self.tensors, offsets):
            h += _str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", x) for x in ne)
            h += struct.pack("<IQ", t, o)
        data_off = (len(h) + align - 1) // align * align
        return h, offsets, data_off

    def to_bytes(self) -> bytes:
        h, offsets, data_off = self.layout()
        out = bytearray(h)
        out += b"\0" * (data_off - len(h))
        for (_, _, _, data), o in zip(self.tensors, offsets):
            out += b"\0" * (data_off + o - len(out))
            out += data
        return bytes(out)

    def write(self, path: Path) -> Path:
        Path(path).write_bytes(self.to_bytes())
        return Path(path)

    def expected_table(self) -> list[dict]:
        """What a reader must report per tensor (name, dims, type, offset, size)."""
        _, offsets, _ = self.layout()
        return [{"name": n, "n_dims": len(ne), "ne": list(ne) + [1] * (4 - len(ne)), "type": t, "offset": o,
                 "size": len(d)} for (n, ne, t, d), o in zip(self.tensors, offsets)]


def f32_bytes(a) -> bytes:
    return np.ascontiguousarray(a, dtype="<f4").tobytes()


def f16_bytes(a) -> bytes:
    return np.ascontiguousarray(a, dtype="<f2").tobytes()


def synthetic_model(n_layer: int = 2, n_embd: int = 512, n_vocab: int = 64, head_dim: int = 128,
                    n_expert: int = 16, embd_type: int = 12, norm_type: int = 1, seed: int = 0,
                    alignment: int | None = None) -> tuple[GgufFile, dict]:
    """A small model file with the engine's tensor names. Norm weights are
    stored as `norm_type` (0 F32, 1 F16, 8 Q8_0); the router as F32 for even
    layers and F16 for odd ones; token_embd as Q4_K (12) or Q6_K (14). Returns
    the file and the raw arrays it holds."""
    from qw3_b200 import inputs as I

    rng = np.random.default_rng(seed)
    g = GgufFile(alignment=alignment)
    g.add_meta("general.architecture", STRING, "qwen3moe")
    g.add_meta("qwen3moe.block_count", U32, n_layer)
    g.add_meta("qwen3moe.embedding_length", U32, n_embd)
    g.add_meta("qwen3moe.attention.layer_norm_rms_epsilon", F32, 1e-6)
    g.add_meta("qwen3moe.rope.freq_base", F32, 1e6)
    g.add_meta("tokenizer.ggml.tokens", ARRAY, (STRING, [f"t{i}" for i in range(8)]))
    g.add_meta("tokenizer.ggml.scores", ARRAY, (F32, [0.5] * 8))
    raw: dict = {}
    tab = (I.q4k_table if embd_type == 12 else I.q6k_table)(n_vocab, n_embd, seed + 1)
    g.add_tensor("token_embd.weight", [n_embd, n_vocab], embd_type, tab.tobytes())
    raw["token_embd.weight"] = tab

    def norm(name, n, s):
        w = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        if norm_type == 0:
            data, val = f32_bytes(w), w
        elif norm_type == 1:
            h = w.astype(np.float16)
            data, val = f16_bytes(h), h.astype(np.float32)
        else:
            data, val = q8_0_bytes(w), None
        g.add_tensor(name, [n], norm_type, data)
        raw[name] = (data, val)

    norm("output_norm.weight", n_embd, 0)
    for l in range(n_layer):
        norm(f"blk.{l}.attn_norm.weight", n_embd, 1)
        norm(f"blk.{l}.attn_q_norm.weight", head_dim, 2)
        norm(f"blk.{l}.attn_k_norm.weight", head_dim, 3)
        norm(f"blk.{l}.ffn_norm.weight", n_embd, 4)
        r = (0.05 * rng.standard_normal((n_expert, n_embd))).astype(np.float32)
        if l % 2:
            rh = r.astype(np.float16)
            g.add_tensor(f"blk.{l}.ffn_gate_inp.weight", [n_embd, n_expert], 1, f16_bytes(rh))
            raw[f"blk.{l}.ffn_gate_inp.weight"] = (f16_bytes(rh), rh.astype(np.float32))
        else:
            g.add_tensor(f"blk.{l}.ffn_gate_inp.weight", [n_embd, n_expert], 0, f32_bytes(r))
            raw[f"blk.{l}.ffn_gate_inp.weight"] = (f32_bytes(r), r)
        # A tensor of the layer the path does not read (kept in the file).
        g.add_tensor(f"blk.{l}.attn_q.weight", [n_embd, 32], 0, f32_bytes(rng.standard_normal((32, n_embd))))
    return g, raw


def q8_0_bytes(w) -> bytes:
    """Blocks of 32: fp16 scale d = max|w|/127, then 32 int8 values round(w/d)."""
    w = np.asarray(w, np.float32).reshape(-1, 32)
    out = bytearray()
    for blk in w:
        amax = float(np.max(np.abs(blk)))
        d = np.float16(amax / 127.0 if amax else 0.0)
        q = np.zeros(32, np.int8) if float(d) == 0 else np.clip(np.rint(blk / float(d)), -127, 127).astype(np.int8)
        out += d.tobytes() + q.tobytes()
    return bytes(out)
