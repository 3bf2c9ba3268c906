"""Python mirror of the ds3_cuda C-ABI (include/ds3_cuda.h).

Every function here is a thin ctypes call into qw3_b200/libds3cuda.so with the
same name (minus the ``ds3_cuda_`` prefix), the same argument order and the
same 0 / -1 return convention as the C entry points, which in turn mirror the
reference engine's ``ds3_metal_*`` functions (src/ds3_metal.h). Buffers are
opaque handles (:class:`Buffer`). There is no fallback: if the shared library
is missing or no B200 is present, the calls fail loudly.

Convenience helpers (``upload``, ``download``, ``empty``) move numpy arrays in
and out of device buffers.
"""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB_PATH = PKG / "libds3cuda.so"
HEADER = ROOT / "include" / "ds3_cuda.h"
HEADERS = sorted((ROOT / "include").glob("*.h"))

# ds3_type_t (src/ds3.h:201-216 of the reference)
TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K = 0, 1, 8, 12, 14

TIMER_SLOTS = 16384

_lib = None

_P = C.c_void_p
_U32, _U64, _F, _I, _SZ, _B = C.c_uint32, C.c_uint64, C.c_float, C.c_int, C.c_size_t, C.c_bool

# name -> (restype, argtypes)
_SIGS = {
    "set_device": (_I, [_I]),
    "init": (_I, []),
    "shutdown": (None, []),
    "buffer_alloc": (_P, [_SZ]),
    "buffer_free": (None, [_P]),
    "buffer_from_mmap": (_P, [_P, _SZ]),
    "buffer_view": (_P, [_P, _SZ, _SZ]),
    "buffer_wrap": (_P, [_P, _SZ]),
    "buffer_device_ptr": (_P, [_P]),
    "buffer_size": (_SZ, [_P]),
    "buffer_write": (_I, [_P, _SZ, _P, _SZ]),
    "buffer_read": (_I, [_P, _SZ, _P, _SZ]),
    "buffer_write_async": (_I, [_P, _SZ, _P, _SZ]),
    "buffer_read_async": (_I, [_P, _SZ, _P, _SZ]),
    "rms_norm": (_I, [_P, _P, _P, _U32, _U32, _F]),
    "rope": (_I, [_P, _P, _P, _U32, _U32, _U32, _F]),
    "buffer_copy_f32": (_I, [_P, _P, _SZ]),
    "buffer_zero_f32": (_I, [_P, _SZ]),
    "vec_add_inplace": (_I, [_P, _P, _U32]),
    "vec_add": (_I, [_P, _P, _P, _U32]),
    "gather_rows_f32": (_I, [_P, _P, _P, _U32, _U32, _U32]),
    "scatter_add_weighted_f32": (_I, [_P, _P, _P, _P, _U32, _U32, _U32]),
    "silu_mul_f32": (_I, [_P, _P, _P, _U32]),
    "moe_router_topk_batch": (_I, [_P, _P, _P, _U32, _U32, _U32, _B]),
    "moe_router_topk_batch_tokens": (_I, [_P, _P, _P, _U32, _U32, _U32, _U32, _B]),
    "begin_batch": (_I, []),
    "end_batch": (_I, []),
    "synchronize": (None, []),
    "profile_reset": (None, []),
    "profile_print": (None, [C.c_char_p]),
    "embed_rows": (_I, [_P, _P, _P, _U32, _U32, _U32, _I, _U64]),
    "embed_rms_norm": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _I, _U64, _F]),
    "add_rms_norm": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _F]),
    "qk_norm_rope": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _F, _F, _I]),
    "router_softmax_topk": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _B]),
    "qk_norm_rope_kv": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _F, _F, _I]),
    "kv_cache_write_batch": (_I, [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32, _U32]),
    "swiglu": (_I, [_P, _P, _P, _P, _U32, _U32]),
    "router_logits_topk": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _B]),
    "moe_expert_lists": (_I, [_P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32]),
    "moe_ffn_router": (_I, [_P, _P, _P, _U32, _U32, _U64, _I]),
    "add_rms_norm_router_topk": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _F, _B]),
    "moe_ffn_router_topk": (_I, [_P, _P, _U64, _I, _P, _P, _P, _U32, _U32, _U32, _U32, _B]),
    "moe_ffn_router_topk_noalloc": (_I, [_P, _P, _U64, _I, _P, _P, _P, _U32, _U32, _U32, _U32, _B]),
    "moe_combine_residual": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32]),
    "stream": (_P, []),
    "lane_write": (_I, [_I, _P, _SZ, _P, _SZ]),
    "lane_read": (_I, [_I, _P, _SZ, _P, _SZ]),
    "lane_record": (_I, [_I, _I]),
    "lane_wait": (_I, [_I, _I]),
    "graph_begin": (_I, []),
    "graph_end": (_P, []),
    "graph_launch": (_I, [_P]),
    "graph_free": (None, [_P]),
    "timer_mark": (_I, [_I]),
    "timer_elapsed_ms": (_F, [_I, _I]),
    "profile_enable": (None, [_I]),
    "last_error": (C.c_char_p, []),
    "device_errors": (_U32, []),
    "selftest_bounded_wait": (_I, [_U32]),
    "kernel_binary_version": (_I, []),
    "dequantize_f32": (_I, [_P, _I, _U64, _P]),
    # include/ds3_cuda_gguf.h
    "gguf_open": (_P, [C.c_char_p]),
    "gguf_close": (None, [_P]),
    "gguf_version": (_U32, [_P]),
    "gguf_alignment": (_U32, [_P]),
    "gguf_data_offset": (_U64, [_P]),
    "gguf_n_tensors": (_U64, [_P]),
    "gguf_n_metadata": (_U64, [_P]),
    "gguf_tensor": (_I, [_P, _U64, _P]),
    "gguf_find_tensor": (_I, [_P, C.c_char_p, _P]),
    "gguf_get_string": (_B, [_P, C.c_char_p, C.POINTER(_P), C.POINTER(_SZ)]),
    "gguf_get_u32": (_B, [_P, C.c_char_p, C.POINTER(_U32)]),
    "gguf_get_f32": (_B, [_P, C.c_char_p, C.POINTER(_F)]),
    "path_weights_load": (_P, [_P, _U32, _B]),
    "path_weights_free": (None, [_P]),
}


def header_symbols() -> list[str]:
    """Every ds3_cuda_* function declared in include/*.h."""
    text = "\n".join(h.read_text() for h in HEADERS)
    return sorted(set(re.findall(r"\b(ds3_cuda_[a-z0-9_]+)\s*\(", text)))


def lib() -> C.CDLL:
    """Load libds3cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m qw3_b200.build` "
                "(there is no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, "ds3_cuda_" + name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class Buffer:
    """Opaque device buffer handle (``ds3_cuda_buffer_t *``)."""

    __slots__ = ("handle", "nbytes", "_freed")

    def __init__(self, handle: int, nbytes: int):
        if not handle:
            raise RuntimeError("ds3_cuda buffer allocation failed: " + last_error())
        self.handle = handle
        self.nbytes = nbytes
        self._freed = False

    @property
    def _as_parameter_(self):
        return C.c_void_p(self.handle)

    @property
    def ptr(self) -> int:
        return lib().ds3_cuda_buffer_device_ptr(self.handle) or 0

    def free(self) -> None:
        if not self._freed:
            lib().ds3_cuda_buffer_free(self.handle)
            self._freed = True


def _h(b):
    return None if b is None else (b.handle if isinstance(b, Buffer) else b)


def last_error() -> str:
    v = lib().ds3_cuda_last_error()
    return v.decode() if v else ""


# ---------------------------------------------------------------- lifecycle
def set_device(device: int) -> int:
    return lib().ds3_cuda_set_device(device)


def init() -> int:
    return lib().ds3_cuda_init()


def shutdown() -> None:
    lib().ds3_cuda_shutdown()


# ------------------------------------------------------------------ buffers
def buffer_alloc(nbytes: int) -> Buffer:
    return Buffer(lib().ds3_cuda_buffer_alloc(nbytes), nbytes)


def buffer_free(buf: Buffer) -> None:
    buf.free()


def buffer_from_mmap(host: np.ndarray) -> Buffer:
    host = np.ascontiguousarray(host)
    return Buffer(lib().ds3_cuda_buffer_from_mmap(host.ctypes.data, host.nbytes), host.nbytes)


def buffer_view(base: Buffer, offset: int, nbytes: int) -> Buffer:
    return Buffer(lib().ds3_cuda_buffer_view(_h(base), offset, nbytes), nbytes)


def buffer_wrap(device_ptr: int, nbytes: int) -> Buffer:
    return Buffer(lib().ds3_cuda_buffer_wrap(device_ptr, nbytes), nbytes)


def buffer_write(buf: Buffer, offset: int, host: np.ndarray) -> int:
    host = np.ascontiguousarray(host)
    return lib().ds3_cuda_buffer_write(_h(buf), offset, host.ctypes.data, host.nbytes)


def buffer_read(buf: Buffer, offset: int, host: np.ndarray) -> int:
    assert host.flags["C_CONTIGUOUS"]
    return lib().ds3_cuda_buffer_read(_h(buf), offset, host.ctypes.data, host.nbytes)


def buffer_write_async(buf: Buffer, offset: int, host: np.ndarray) -> int:
    """Enqueue a host->device copy; `host` must stay alive and unchanged until synchronize()."""
    assert host.flags["C_CONTIGUOUS"]
    return lib().ds3_cuda_buffer_write_async(_h(buf), offset, host.ctypes.data, host.nbytes)


def buffer_read_async(buf: Buffer, offset: int, host: np.ndarray) -> int:
    """Enqueue a device->host copy into `host`, valid after synchronize()."""
    assert host.flags["C_CONTIGUOUS"]
    return lib().ds3_cuda_buffer_read_async(_h(buf), offset, host.ctypes.data, host.nbytes)


def lane_write(lane: int, buf: Buffer, offset: int, host: np.ndarray) -> int:
    """Enqueue a host->device copy on copy lane `lane` (0 = the ops' stream)."""
    assert host.flags["C_CONTIGUOUS"]
    return lib().ds3_cuda_lane_write(lane, _h(buf), offset, host.ctypes.data, host.nbytes)


def lane_read(lane: int, buf: Buffer, offset: int, host: np.ndarray) -> int:
    """Enqueue a device->host copy on copy lane `lane`."""
    assert host.flags["C_CONTIGUOUS"]
    return lib().ds3_cuda_lane_read(lane, _h(buf), offset, host.ctypes.data, host.nbytes)


def lane_record(lane: int, slot: int) -> int:
    return lib().ds3_cuda_lane_record(lane, slot)


def lane_wait(lane: int, slot: int) -> int:
    return lib().ds3_cuda_lane_wait(lane, slot)


def upload(host: np.ndarray) -> Buffer:
    host = np.ascontiguousarray(host)
    b = buffer_alloc(max(host.nbytes, 1))
    if host.nbytes and buffer_write(b, 0, host) != 0:
        raise RuntimeError("buffer_write failed: " + last_error())
    return b


def empty(nbytes: int) -> Buffer:
    return buffer_alloc(max(int(nbytes), 1))


def download(buf: Buffer, dtype, shape) -> np.ndarray:
    out = np.empty(shape, dtype=dtype)
    if out.nbytes and buffer_read(buf, 0, out) != 0:
        raise RuntimeError("buffer_read failed: " + last_error())
    return out


# ------------------------------------------------------ ops (Metal mirror)
def rms_norm(x, weight, out, n, n_rows, eps) -> int:
    return lib().ds3_cuda_rms_norm(_h(x), _h(weight), _h(out), n, n_rows, eps)


def rope(src, dst, positions, n_heads, head_dim, n_rows, theta_base) -> int:
    return lib().ds3_cuda_rope(_h(src), _h(dst), _h(positions), n_heads, head_dim, n_rows, theta_base)


def buffer_copy_f32(src, dst, nbytes) -> int:
    return lib().ds3_cuda_buffer_copy_f32(_h(src), _h(dst), nbytes)


def buffer_zero_f32(buf, nbytes) -> int:
    return lib().ds3_cuda_buffer_zero_f32(_h(buf), nbytes)


def vec_add_inplace(acc, addend, n) -> int:
    return lib().ds3_cuda_vec_add_inplace(_h(acc), _h(addend), n)


def vec_add(a, b, c, n) -> int:
    return lib().ds3_cuda_vec_add(_h(a), _h(b), _h(c), n)


def gather_rows_f32(src, ids, dst, n_cols, count, offset) -> int:
    return lib().ds3_cuda_gather_rows_f32(_h(src), _h(ids), _h(dst), n_cols, count, offset)


def scatter_add_weighted_f32(src, scores, ids, dst, n_cols, count, offset) -> int:
    return lib().ds3_cuda_scatter_add_weighted_f32(_h(src), _h(scores), _h(ids), _h(dst), n_cols, count, offset)


def silu_mul_f32(gate, up, out, n) -> int:
    return lib().ds3_cuda_silu_mul_f32(_h(gate), _h(up), _h(out), n)


def moe_router_topk_batch(logits, indices, scores, n_layers, n_expert, n_used, norm_topk_prob) -> int:
    return lib().ds3_cuda_moe_router_topk_batch(_h(logits), _h(indices), _h(scores), n_layers, n_expert,
                                                n_used, bool(norm_topk_prob))


def moe_router_topk_batch_tokens(logits, indices, scores, n_layers, n_tokens, n_expert, n_used,
                                 norm_topk_prob) -> int:
    return lib().ds3_cuda_moe_router_topk_batch_tokens(_h(logits), _h(indices), _h(scores), n_layers,
                                                       n_tokens, n_expert, n_used, bool(norm_topk_prob))


def begin_batch() -> int:
    return lib().ds3_cuda_begin_batch()


def end_batch() -> int:
    return lib().ds3_cuda_end_batch()


def synchronize() -> None:
    lib().ds3_cuda_synchronize()


def profile_reset() -> None:
    lib().ds3_cuda_profile_reset()


def profile_print(label: str) -> None:
    lib().ds3_cuda_profile_print(label.encode())


def profile_enable(on: bool) -> None:
    lib().ds3_cuda_profile_enable(1 if on else 0)


# ---------------------------------------------------------------- fused ops
def embed_rows(table, ids, out, n_ids, n_cols, n_vocab, type_, row_stride) -> int:
    return lib().ds3_cuda_embed_rows(_h(table), _h(ids), _h(out), n_ids, n_cols, n_vocab, type_, row_stride)


def embed_rms_norm(table, ids, weight, hidden_out, norm_out, n_ids, n_cols, n_vocab, type_, row_stride,
                   eps) -> int:
    return lib().ds3_cuda_embed_rms_norm(_h(table), _h(ids), _h(weight), _h(hidden_out), _h(norm_out), n_ids,
                                         n_cols, n_vocab, type_, row_stride, eps)


def add_rms_norm(x, residual, weight, sum_out, norm_out, n, n_rows, eps) -> int:
    return lib().ds3_cuda_add_rms_norm(_h(x), _h(residual), _h(weight), _h(sum_out), _h(norm_out), n, n_rows, eps)


def qk_norm_rope(q, k, q_w, k_w, positions, n_rows, n_q_heads, n_kv_heads, head_dim, theta_base, eps,
                 storage=TYPE_F32) -> int:
    return lib().ds3_cuda_qk_norm_rope(_h(q), _h(k), _h(q_w), _h(k_w), _h(positions), n_rows, n_q_heads,
                                       n_kv_heads, head_dim, theta_base, eps, storage)


def qk_norm_rope_kv(q, k, v, q_w, k_w, positions, k_cache, v_cache, n_rows, n_q_heads, n_kv_heads, head_dim,
                    max_seq_len, theta_base, eps, storage=TYPE_F32) -> int:
    return lib().ds3_cuda_qk_norm_rope_kv(_h(q), _h(k), _h(v), _h(q_w), _h(k_w), _h(positions), _h(k_cache),
                                          _h(v_cache), n_rows, n_q_heads, n_kv_heads, head_dim, max_seq_len,
                                          theta_base, eps, storage)


def kv_cache_write_batch(k, v, k_cache, v_cache, seq_pos, n_tokens, max_seq_len, n_q_heads, n_kv_heads,
                         head_dim) -> int:
    return lib().ds3_cuda_kv_cache_write_batch(_h(k), _h(v), _h(k_cache), _h(v_cache), seq_pos, n_tokens,
                                               max_seq_len, n_q_heads, n_kv_heads, head_dim)


def router_softmax_topk(logits, probs_out, idx, scores, n_tokens, n_expert, n_used, norm_topk_prob) -> int:
    return lib().ds3_cuda_router_softmax_topk(_h(logits), _h(probs_out), _h(idx), _h(scores), n_tokens,
                                              n_expert, n_used, bool(norm_topk_prob))


def router_logits_topk(x, w_router, logits_out, idx, scores, n_tokens, n_embd, n_expert, n_used,
                       norm_topk_prob=True) -> int:
    return lib().ds3_cuda_router_logits_topk(_h(x), _h(w_router), _h(logits_out), _h(idx), _h(scores), n_tokens,
                                             n_embd, n_expert, n_used, bool(norm_topk_prob))


def add_rms_norm_router_topk(x, residual, norm_weight, w_router, sum_out, norm_out, logits_out, idx, scores,
                             n_tokens, n_embd, n_expert, n_used, eps, norm_topk_prob=True) -> int:
    return lib().ds3_cuda_add_rms_norm_router_topk(_h(x), _h(residual), _h(norm_weight), _h(w_router), _h(sum_out),
                                                   _h(norm_out), _h(logits_out), _h(idx), _h(scores), n_tokens,
                                                   n_embd, n_expert, n_used, eps, bool(norm_topk_prob))


def moe_ffn_router(input_, w_gate_inp, gate_logits, n_embd, n_expert, router_row_stride, router_type) -> int:
    return lib().ds3_cuda_moe_ffn_router(_h(input_), _h(w_gate_inp), _h(gate_logits), n_embd, n_expert,
                                         router_row_stride, router_type)


def moe_ffn_router_topk(input_, w_gate_inp, router_row_stride, router_type, gate_logits, idx, scores, n_tokens,
                        n_embd, n_expert, n_used, norm_topk_prob=True) -> int:
    return lib().ds3_cuda_moe_ffn_router_topk(_h(input_), _h(w_gate_inp), router_row_stride, router_type,
                                              _h(gate_logits), _h(idx), _h(scores), n_tokens, n_embd, n_expert,
                                              n_used, bool(norm_topk_prob))


def moe_ffn_router_topk_noalloc(input_, w_gate_inp, router_row_stride, router_type, gate_logits, idx, scores,
                                n_tokens, n_embd, n_expert, n_used, norm_topk_prob=True) -> int:
    """moe_ffn_router_topk without any device allocation (fixed in-library scratch)."""
    return lib().ds3_cuda_moe_ffn_router_topk_noalloc(_h(input_), _h(w_gate_inp), router_row_stride, router_type,
                                                      _h(gate_logits), _h(idx), _h(scores), n_tokens, n_embd,
                                                      n_expert, n_used, bool(norm_topk_prob))


def moe_expert_lists(idx, scores, counts, ids, gscores, slot_of, n_tokens, n_expert, n_used, cap) -> int:
    return lib().ds3_cuda_moe_expert_lists(_h(idx), _h(scores), _h(counts), _h(ids), _h(gscores), _h(slot_of),
                                           n_tokens, n_expert, n_used, cap)


def swiglu(gate, up, row_weight, out, n_rows, n_cols) -> int:
    return lib().ds3_cuda_swiglu(_h(gate), _h(up), _h(row_weight), _h(out), n_rows, n_cols)


def moe_combine_residual(y, y_rows, w, residual, out, n_tokens, n_used, n_cols) -> int:
    return lib().ds3_cuda_moe_combine_residual(_h(y), _h(y_rows), _h(w), _h(residual), _h(out), n_tokens,
                                               n_used, n_cols)


# ------------------------------------------------- streams / graphs / timers
def stream() -> int:
    return lib().ds3_cuda_stream() or 0


def graph_begin() -> int:
    return lib().ds3_cuda_graph_begin()


def graph_end() -> int:
    g = lib().ds3_cuda_graph_end()
    if not g:
        raise RuntimeError("graph_end failed: " + last_error())
    return g


def graph_launch(g) -> int:
    return lib().ds3_cuda_graph_launch(g)


def graph_free(g) -> None:
    lib().ds3_cuda_graph_free(g)


def timer_mark(slot: int) -> int:
    return lib().ds3_cuda_timer_mark(slot)


def timer_elapsed_ms(a: int, b: int) -> float:
    return lib().ds3_cuda_timer_elapsed_ms(a, b)


def device_errors() -> int:
    return lib().ds3_cuda_device_errors()


def kernel_binary_version() -> int:
    return lib().ds3_cuda_kernel_binary_version()


def selftest_bounded_wait(polls: int = 1000) -> int:
    return lib().ds3_cuda_selftest_bounded_wait(polls)


def dequantize_f32(src, type_, n_elements, dst) -> int:
    return lib().ds3_cuda_dequantize_f32(_h(src), type_, n_elements, _h(dst))


# ---------------------------------------------------------------------------
# GGUF reader and path-weight binding (include/ds3_cuda_gguf.h)
# ---------------------------------------------------------------------------

class GgufTensorInfo(C.Structure):
    """ds3_cuda_gguf_tensor_t"""

    _fields_ = [("name", _P), ("name_len", _U64), ("n_dims", _U32), ("ne", _U64 * 4), ("nb", _U64 * 4),
                ("type", _U32), ("offset", _U64), ("size", _U64), ("data", _P)]

    def as_dict(self) -> dict:
        return {"name": C.string_at(self.name, self.name_len).decode(), "n_dims": self.n_dims,
                "ne": list(self.ne), "nb": list(self.nb), "type": self.type, "offset": self.offset,
                "size": self.size}


class PathWeightsC(C.Structure):
    """ds3_cuda_path_weights_t"""

    _fields_ = [("n_layer", _U32), ("n_embd", _U32), ("n_vocab", _U32), ("head_dim", _U32), ("n_expert", _U32),
                ("token_embd_type", _U32), ("token_embd_row_stride", _U64), ("token_embd", _P),
                ("output_norm", _P), ("attn_norm", C.POINTER(_P)), ("attn_q_norm", C.POINTER(_P)),
                ("attn_k_norm", C.POINTER(_P)), ("ffn_norm", C.POINTER(_P)), ("ffn_gate_inp", C.POINTER(_P))]


class Gguf:
    """An open GGUF file (ds3_cuda_gguf_open); close() or use as a context manager."""

    def __init__(self, path):
        self.handle = lib().ds3_cuda_gguf_open(str(path).encode())
        if not self.handle:
            raise OSError(last_error())

    def close(self) -> None:
        if self.handle:
            lib().ds3_cuda_gguf_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def version(self) -> int:
        return lib().ds3_cuda_gguf_version(self.handle)

    @property
    def alignment(self) -> int:
        return lib().ds3_cuda_gguf_alignment(self.handle)

    @property
    def data_offset(self) -> int:
        return lib().ds3_cuda_gguf_data_offset(self.handle)

    @property
    def n_metadata(self) -> int:
        return lib().ds3_cuda_gguf_n_metadata(self.handle)

    def tensors(self) -> list[dict]:
        out = []
        for i in range(lib().ds3_cuda_gguf_n_tensors(self.handle)):
            t = GgufTensorInfo()
            assert lib().ds3_cuda_gguf_tensor(self.handle, i, C.byref(t)) == 0
            out.append(t.as_dict())
        return out

    def find(self, name: str) -> dict | None:
        t = GgufTensorInfo()
        if lib().ds3_cuda_gguf_find_tensor(self.handle, name.encode(), C.byref(t)) != 0:
            return None
        return t.as_dict()

    def get_string(self, key: str) -> bytes | None:
        p, n = _P(), _SZ()
        if not lib().ds3_cuda_gguf_get_string(self.handle, key.encode(), C.byref(p), C.byref(n)):
            return None
        return C.string_at(p.value, n.value)

    def get_u32(self, key: str) -> int | None:
        v = _U32()
        return v.value if lib().ds3_cuda_gguf_get_u32(self.handle, key.encode(), C.byref(v)) else None

    def get_f32(self, key: str) -> float | None:
        v = _F()
        return v.value if lib().ds3_cuda_gguf_get_f32(self.handle, key.encode(), C.byref(v)) else None


class PathWeights:
    """Device tensors of the fused path bound from a GGUF file
    (ds3_cuda_path_weights_load). Buffer fields are borrowed handles, freed
    together by free()."""

    def __init__(self, gguf: Gguf, n_layer: int, require_qk_norm: bool = True):
        self.handle = lib().ds3_cuda_path_weights_load(gguf.handle, n_layer, require_qk_norm)
        if not self.handle:
            raise RuntimeError(last_error())
        self.c = C.cast(self.handle, C.POINTER(PathWeightsC)).contents

    @staticmethod
    def _buf(h, nbytes: int) -> "Buffer | None":
        return _Borrowed(h, nbytes) if h else None

    def layer(self, name: str, i: int, nbytes: int) -> "Buffer | None":
        return self._buf(getattr(self.c, name)[i], nbytes)

    def free(self) -> None:
        if self.handle:
            lib().ds3_cuda_path_weights_free(self.handle)
            self.handle = None


class _Borrowed(Buffer):
    """A buffer owned by something else (freeing it is a no-op)."""

    def __init__(self, handle: int, nbytes: int):
        super().__init__(handle, nbytes)

    def free(self) -> None:
        pass
