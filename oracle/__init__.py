"""ctypes front-end for the CPU oracles.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py's cpu_baseline / reference legs. The product
(qw3_b200/) never imports this package.

Two libraries share one signature set (oracle/ds3_oracle.h):
  * ``port()``      — oracle/libds3oracle.so, the restatement (ds3o_*),
  * ``reference()`` — oracle/_ref/libds3ref.so, the unmodified reference
                      kernels driven by oracle/ref_harness.c (ds3r_*); None
                      when it has not been built (it needs the reference
                      sources at build time).
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "libds3oracle.so"
REF_LIB = HERE / "_ref" / "libds3ref.so"

_P, _I, _I64, _U64, _F = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_float

_SIGS = {
    "embed_rows": (_I, [_P, _I, _U64, _I64, _P, _I64, _I64, _P, _I]),
    "embed_rms_norm": (_I, [_P, _I, _U64, _I64, _P, _I64, _I64, _P, _F, _P, _P, _I]),
    "rms_norm_rows": (None, [_P, _P, _F, _I, _I64, _P, _I]),
    "add_rms_norm": (None, [_P, _P, _P, _F, _I, _I64, _P, _P, _I]),
    "qk_norm_rope": (None, [_P, _P, _P, _P, _P, _I64, _I, _I, _I, _F, _F, _I]),
    "rope_rows": (None, [_P, _P, _P, _I, _I, _I64, _F, _I]),
    "router_softmax_topk": (None, [_P, _I64, _I, _I, _I, _P, _P, _P, _I]),
    "swiglu": (None, [_P, _P, _P, _P, _I64, _I64, _I]),
    "moe_combine_residual": (None, [_P, _P, _P, _P, _P, _I64, _I, _I64, _I]),
    "max_threads": (_I, []),
    "router_logits": (None, [_P, _P, _I64, _I, _I, _P, _I]),
}
_PORT_ONLY = {
    "dequant_row": (_I, [_I, _P, _I64, _P]),
    "softmax": (None, [_P, _I]),
    "topk": (None, [_P, _I, _I, _P, _P]),
    "rope_token": (None, [_P, _P, _I, _I, _I, _I, _F]),
    "rms_norm": (None, [_P, _P, _F, _I, _P]),
    "scatter_add_weighted": (None, [_P, _P, _P, _P, _I64, _I64, _I64]),
    "gather_rows": (None, [_P, _P, _P, _I64, _I64, _I64]),
    "fp16_to_fp32": (_F, [C.c_uint16]),
    "kv_cache_write": (None, [_P, _P, _P, _I64, _I64, _I64, _P, _P]),
    "moe_expert_lists": (_I, [_P, _P, _I64, _I, _I, _I64, _P, _P, _P, _P]),
}


def reference_dir() -> str:
    """The reference checkout the Makefile builds from: DS3_REFERENCE_DIR if
    set, else the Makefile's default REF (a sibling of the repository)."""
    env = os.environ.get("DS3_REFERENCE_DIR")
    if env:
        return env
    out = subprocess.run(["make", "-s", "-C", str(HERE), "print-ref"], capture_output=True, text=True)
    return out.stdout.strip()


def build(ref_dir: str | None = None, quiet: bool = True) -> None:
    """Compile the oracles with oracle/Makefile (the reference leg only when
    the reference tree is present)."""
    targets = ["oracle"]
    ref = ref_dir or reference_dir()
    if Path(ref, "src", "ds3_reference.c").exists():
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF={ref}", *targets], check=True,
                   capture_output=quiet)


def _arr(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _p(a):
    return None if a is None else a.ctypes.data


class Oracle:
    """numpy interface over one oracle library."""

    def __init__(self, path: Path, prefix: str, extra: dict | None = None):
        self.path = path
        self.kind = "port" if prefix == "ds3o_" else "reference"
        L = C.CDLL(str(path))
        sigs = dict(_SIGS)
        if extra:
            sigs.update(extra)
        for name, (res, args) in sigs.items():
            fn = getattr(L, prefix + name)
            fn.restype, fn.argtypes = res, args
            setattr(self, "_" + name, fn)
        self.lib = L

    def max_threads(self) -> int:
        return self._max_threads()

    # ------------------------------------------------------------ embedding
    def embed_rows(self, table: np.ndarray, type_: int, row_stride: int, n_vocab: int, ids, n_cols: int,
                   nthreads: int = 1):
        ids = _arr(ids, np.int32)
        out = np.empty((ids.size, n_cols), np.float32)
        rc = self._embed_rows(_p(table), type_, row_stride, n_vocab, _p(ids), ids.size, n_cols, _p(out),
                              nthreads)
        return rc, out

    def embed_rms_norm(self, table, type_, row_stride, n_vocab, ids, n_cols, w, eps, nthreads=1):
        ids = _arr(ids, np.int32)
        w = _arr(w, np.float32)
        hid = np.empty((ids.size, n_cols), np.float32)
        nrm = np.empty_like(hid)
        rc = self._embed_rms_norm(_p(table), type_, row_stride, n_vocab, _p(ids), ids.size, n_cols, _p(w), eps,
                                  _p(hid), _p(nrm), nthreads)
        return rc, hid, nrm

    # ---------------------------------------------------------------- norms
    def rms_norm_rows(self, x, w, eps, nthreads=1):
        x = _arr(x, np.float32)
        w = _arr(w, np.float32)
        n = w.size
        out = np.empty_like(x)
        self._rms_norm_rows(_p(x), _p(w), eps, n, x.size // n, _p(out), nthreads)
        return out

    def add_rms_norm(self, x, r, w, eps, nthreads=1):
        x, r, w = _arr(x, np.float32), _arr(r, np.float32), _arr(w, np.float32)
        n = w.size
        s = np.empty_like(x)
        o = np.empty_like(x)
        self._add_rms_norm(_p(x), _p(r), _p(w), eps, n, x.size // n, _p(s), _p(o), nthreads)
        return s, o

    # ----------------------------------------------------------------- rope
    def qk_norm_rope(self, q, k, q_w, k_w, pos, theta, eps, nthreads=1):
        """q [T,nq,hd], k [T,nk,hd] (copies are rotated and returned)."""
        q = np.array(q, dtype=np.float32, order="C", copy=True)
        k = np.array(k, dtype=np.float32, order="C", copy=True)
        pos = _arr(pos, np.int32)
        T, nq, hd = q.shape
        nk = k.shape[1]
        self._qk_norm_rope(_p(q), _p(k), _p(_arr(q_w, np.float32)), _p(_arr(k_w, np.float32)), _p(pos), T, nq, nk,
                           hd, theta, eps, nthreads)
        return q, k

    def rope_rows(self, x, pos, theta, nthreads=1):
        """x [T, n_heads, hd] -> rotated copy."""
        x = _arr(x, np.float32)
        T, nh, hd = x.shape
        out = np.empty_like(x)
        self._rope_rows(_p(x), _p(out), _p(_arr(pos, np.int32)), nh, hd, T, theta, nthreads)
        return out

    # --------------------------------------------------------------- router
    def router(self, logits, n_used, norm=True, nthreads=1):
        logits = _arr(logits, np.float32)
        T, E = logits.shape
        probs = np.empty_like(logits)
        idx = np.empty((T, n_used), np.int32)
        sc = np.empty((T, n_used), np.float32)
        self._router_softmax_topk(_p(logits), T, E, n_used, 1 if norm else 0, _p(probs), _p(idx), _p(sc), nthreads)
        return probs, idx, sc

    def router_logits(self, x, W, nthreads=1):
        """x [T, n_embd], W [n_expert, n_embd] -> logits [T, n_expert]."""
        x, W = _arr(x, np.float32), _arr(W, np.float32)
        T, K = x.shape
        E = W.shape[0]
        out = np.empty((T, E), np.float32)
        self._router_logits(_p(x), _p(W), T, K, E, _p(out), nthreads)
        return out

    # ----------------------------------------------------------------- moe
    def swiglu(self, gate, up, row_w=None, nthreads=1):
        gate, up = _arr(gate, np.float32), _arr(up, np.float32)
        R, Cc = gate.shape
        out = np.empty_like(gate)
        rw = None if row_w is None else _arr(row_w, np.float32)
        self._swiglu(_p(gate), _p(up), _p(rw), _p(out), R, Cc, nthreads)
        return out

    def combine(self, y, w, residual, y_rows=None, nthreads=1):
        y, w, residual = _arr(y, np.float32), _arr(w, np.float32), _arr(residual, np.float32)
        T, K = w.shape
        Cc = residual.shape[1]
        out = np.empty_like(residual)
        yr = None if y_rows is None else _arr(y_rows, np.int32)
        self._moe_combine_residual(_p(y), _p(yr), _p(w), _p(residual), _p(out), T, K, Cc, nthreads)
        return out


def kv_cache_write(O: Oracle, k, v, cache_k, cache_v, seq_pos=0, row_of=None):
    """Port oracle only: writes fp16 rows of k/v ([T, n_kv, hd] fp32) into the
    uint16 caches ([max_seq, n_kv, hd]) in place."""
    k, v = _arr(k, np.float32), _arr(v, np.float32)
    T = k.shape[0]
    row = k.size // max(T, 1)
    ro = None if row_of is None else _arr(row_of, np.int32)
    assert cache_k.dtype == np.uint16 and cache_k.flags["C_CONTIGUOUS"] and cache_v.flags["C_CONTIGUOUS"]
    O._kv_cache_write(_p(k), _p(v), _p(ro), seq_pos, T, row, _p(cache_k), _p(cache_v))


def moe_expert_lists(O: Oracle, idx, scores, n_expert, cap, fill_ids=-7, fill_scores=np.nan):
    """Port oracle only: (rc, counts, ids, gscores, slot_of); unwritten slots keep the fill values."""
    idx, scores = _arr(idx, np.int32), _arr(scores, np.float32)
    T, K = idx.shape
    counts = np.zeros(n_expert, np.int32)
    ids = np.full(n_expert * cap, fill_ids, np.int32)
    gs = np.full(n_expert * cap, fill_scores, np.float32)
    slot = np.empty(T * K, np.int32)
    rc = O._moe_expert_lists(_p(idx), _p(scores), T, K, n_expert, cap, _p(counts), _p(ids), _p(gs), _p(slot))
    return rc, counts, ids, gs, slot


_port = None
_ref = None


def port() -> Oracle:
    global _port
    if _port is None:
        if not PORT_LIB.exists():
            build()
        _port = Oracle(PORT_LIB, "ds3o_", _PORT_ONLY)
    return _port


def reference() -> Oracle | None:
    global _ref
    if _ref is None and REF_LIB.exists():
        _ref = Oracle(REF_LIB, "ds3r_")
    return _ref


REF_GGUF_LIB = HERE / "_ref" / "libds3gguf.so"
_ref_gguf = None


def reference_gguf(path) -> dict | None:
    """Header and tensor table of `path` as parsed by the unmodified reference
    reader (oracle/_ref/libds3gguf.so; None when it has not been built), or
    {"error": True} when that reader rejects the file. Same keys as
    oracle.gguf.parse() minus metadata and strides."""
    global _ref_gguf
    if _ref_gguf is None:
        if not REF_GGUF_LIB.exists():
            return None
        L = C.CDLL(str(REF_GGUF_LIB))
        L.ds3rg_open.restype, L.ds3rg_open.argtypes = _P, [C.c_char_p]
        L.ds3rg_close.restype, L.ds3rg_close.argtypes = None, [_P]
        L.ds3rg_header.restype, L.ds3rg_header.argtypes = None, [_P, _P]
        L.ds3rg_tensor.restype, L.ds3rg_tensor.argtypes = _I, [_P, _U64, C.c_char_p, C.c_size_t, _P]
        _ref_gguf = L
    L = _ref_gguf
    h = L.ds3rg_open(str(path).encode())
    if not h:
        return {"error": True}
    try:
        hd = np.zeros(5, np.uint64)
        L.ds3rg_header(h, hd.ctypes.data)
        table = []
        name = C.create_string_buffer(512)
        for i in range(int(hd[2])):
            o = np.zeros(10, np.uint64)
            assert L.ds3rg_tensor(h, i, name, 512, o.ctypes.data) == 0
            n_dims = int(o[0])
            table.append({"name": name.value.decode(), "n_dims": n_dims,
                          "ne": [int(o[1 + d]) if d < n_dims else 1 for d in range(4)], "type": int(o[5]),
                          "offset": int(o[6]), "size": int(o[7]), "data_at": int(o[8])})
        return {"version": int(hd[0]), "alignment": int(hd[1]), "n_metadata": int(hd[3]),
                "data_offset": int(hd[4]), "tensors": table}
    finally:
        L.ds3rg_close(h)
