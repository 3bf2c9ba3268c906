"""Router projection fused with softmax/top-k (ds3_cuda_router_logits_topk):
logits bit-exact with the reference's sequential vec_matmul (restated in the
oracle), top-k indices exact, scores within the fp32 tolerance."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_bitexact, assert_close
from qw3_b200 import inputs as I

pytestmark = pytest.mark.gpu


@pytest.fixture
def up(ds3):
    keep = []

    def f(a):
        b = ds3.upload(np.ascontiguousarray(a))
        keep.append(b)
        return b

    yield f
    for b in keep:
        b.free()
    assert ds3.device_errors() == 0


@pytest.mark.parametrize("T,K,E,n_used,with_logits", [(512, 2048, 128, 8, True), (512, 2048, 128, 8, False),
                                                      (2, 2048, 128, 8, False), (31, 2048, 128, 8, True),
                                                      (97, 2048, 128, 8, False), (129, 2048, 128, 8, True),
                                                      (150, 512, 128, 8, True), (300, 2048, 128, 32, True),
                                                      (1, 2048, 128, 8, True), (67, 1024, 128, 8, True),
                                                      (13, 100, 64, 4, True), (5, 2048, 32, 8, True),
                                                      (70, 2080, 128, 8, True), (1000, 2048, 128, 8, True)])
def test_router_logits_topk(ds3, up, port, T, K, E, n_used, with_logits):
    x = I.normal(T + K, (T, K))
    W = I.normal(E + 7, (E, K), 0.0, 0.05)
    lg = port.router_logits(x, W, 8)
    _, want_i, want_s = port.router(lg, n_used, True)
    lb = up(np.zeros((T, E), np.float32)) if with_logits else None
    ib, sb = up(np.zeros((T, n_used), np.int32)), up(np.zeros((T, n_used), np.float32))
    rc = ds3.router_logits_topk(up(x), up(W), lb, ib, sb, T, K, E, n_used, True)
    assert rc == 0, ds3.last_error()
    if with_logits:
        assert_bitexact(ds3.download(lb, np.float32, (T, E)), lg, "logits")
    assert_bitexact(ds3.download(ib, np.int32, (T, n_used)), want_i, "top-k")
    assert_close(ds3.download(sb, np.float32, (T, n_used)), want_s, what="scores")


def test_router_logits_topk_needs_logits_off_the_fast_path(ds3, up):
    x, W = I.normal(1, (4, 100)), I.normal(2, (64, 100))
    ib, sb = up(np.zeros((4, 4), np.int32)), up(np.zeros((4, 4), np.float32))
    assert ds3.router_logits_topk(up(x), up(W), None, ib, sb, 4, 100, 64, 4, True) == -1
    # 128 experts but n_embd not a multiple of 64: also the general path.
    x2, W2 = I.normal(3, (4, 2080)), I.normal(4, (128, 2080))
    ib2, sb2 = up(np.zeros((4, 8), np.int32)), up(np.zeros((4, 8), np.float32))
    assert ds3.router_logits_topk(up(x2), up(W2), None, ib2, sb2, 4, 2080, 128, 8, True) == -1


# ------------------------------------------------- router weight in its stored type
F32, F16, Q80, Q4K, Q6K = 0, 1, 8, 12, 14


def stored_router(type_, E, K, seed, pad=0):
    """Router weight [E, K] stored as `type_` (GGUF row layout), rows `pad`
    bytes longer than their data when pad > 0. Returns (bytes [E, stride], stride)."""
    g = I.rng(seed)
    if type_ == F32:
        rows = I.normal(seed, (E, K), 0.0, 0.05).view(np.uint8)
    elif type_ == F16:
        rows = I.normal(seed, (E, K), 0.0, 0.05).astype(np.float16).view(np.uint8)
    elif type_ == Q80:
        rows = g.integers(0, 256, (E, K // 32, 34), dtype=np.uint8)
        rows[:, :, 0:2] = g.uniform(0, 0.002, (E, K // 32, 1)).astype(np.float16).view(np.uint8)
        rows = rows.reshape(E, -1)
    elif type_ == Q4K:
        # Small super-block scales keep the logits in a range where softmax
        # leaves no exact ties among the top 8 (ties are excluded from parity).
        rows = I.q4k_table(E, K, seed).reshape(E, K // 256, 144)
        rows[:, :, 0:4] = g.uniform(0, 2e-4, (E, K // 256, 2)).astype(np.float16).view(np.uint8)
        rows = rows.reshape(E, -1)
    else:
        rows = I.q6k_table(E, K, seed).reshape(E, K // 256, 210)
        rows[:, :, 208:210] = g.uniform(0, 2e-4, (E, K // 256, 1)).astype(np.float16).view(np.uint8)
        rows = rows.reshape(E, -1)
    if pad:
        rows = np.concatenate([rows, np.zeros((E, pad), np.uint8)], axis=1)
    return np.ascontiguousarray(rows), rows.shape[1]


@pytest.mark.parametrize("type_,T,pad", [(F32, 512, 0), (F16, 512, 0), (Q80, 512, 0), (F16, 64, 0), (Q80, 1, 0),
                                         (F32, 37, 16), (F16, 9, 48), (Q4K, 70, 0), (Q6K, 3, 0)])
def test_moe_ffn_router_stored_types(ds3, up, port, type_, T, pad):
    """Logits bit-exact with the reference's vec_matmul over the dequantised
    weight, for each stored type (the fused top-8 path and the Metal-shaped
    one-token entry point)."""
    E, K, n_used = 128, 2048, 8
    x = I.normal(31 + T, (T, K))
    wb, stride = stored_router(type_, E, K, 40 + type_, pad)
    _, Wf = port.embed_rows(wb, type_, stride, E, np.arange(E, dtype=np.int32), K)
    lg = port.router_logits(x, Wf, 8)
    _, want_i, want_s = port.router(lg, n_used, True)
    xb, wbuf = up(x), up(wb)
    lb = up(np.zeros((T, E), np.float32))
    ib, sb = up(np.zeros((T, n_used), np.int32)), up(np.zeros((T, n_used), np.float32))
    assert ds3.moe_ffn_router_topk(xb, wbuf, stride, type_, lb, ib, sb, T, K, E, n_used, True) == 0, ds3.last_error()
    assert_bitexact(ds3.download(lb, np.float32, (T, E)), lg, "logits")
    assert_bitexact(ds3.download(ib, np.int32, (T, n_used)), want_i, "top-8")
    assert_close(ds3.download(sb, np.float32, (T, n_used)), want_s, what="scores")
    # Without the logits buffer (fast path), then the one-token Metal-shaped entry.
    assert ds3.moe_ffn_router_topk(xb, wbuf, stride, type_, None, ib, sb, T, K, E, n_used, True) == 0
    assert_bitexact(ds3.download(ib, np.int32, (T, n_used)), want_i, "top-8 (no logits)")
    one = up(np.zeros(E, np.float32))
    assert ds3.moe_ffn_router(xb, wbuf, one, K, E, stride, type_) == 0, ds3.last_error()
    assert_bitexact(ds3.download(one, np.float32, (E,)), lg[0], "one-token logits")


def test_moe_ffn_router_argument_errors(ds3, up):
    x = up(I.normal(1, (2, 2048)))
    w, stride = stored_router(F16, 128, 2048, 5)
    wb = up(w)
    lb = up(np.zeros((2, 128), np.float32))
    assert ds3.moe_ffn_router(x, wb, lb, 2048, 128, stride - 2, F16) == -1  # stride shorter than a row
    assert ds3.moe_ffn_router(x, wb, lb, 2048, 128, stride, 7) == -1       # unknown type
    assert ds3.moe_ffn_router(x, wb, lb, 2048, 256, stride, F16) == -1     # weight buffer too small
    assert ds3.moe_ffn_router_topk(x, wb, stride, F16, lb, None, None, 2, 2048, 128, 8, True) == -1


@pytest.mark.parametrize("T,K,in_place", [(64, 2048, False), (64, 2048, True), (1, 2048, False), (512, 2048, False),
                                          (150, 2048, True), (300, 2048, False), (33, 256, True),
                                          (37, 1024, True), (9, 128, False)])
def test_add_rms_norm_router_topk(ds3, up, port, T, K, in_place):
    """The decode FFN entry in one launch: the sum bit-exact with the oracle,
    the normed rows bit-identical to add_rms_norm's (and within tolerance of
    the oracle), the logits bit-exact with the reference's vec_matmul over
    those normed rows, top-8 exact."""
    E, n_used = 128, 8
    x, r = I.normal(60 + T, (T, K)), I.normal(61 + T, (T, K))
    w, W = I.gamma(K, 62), I.normal(63, (E, K), 0.0, 0.05)
    xb, rb, wb, Wb = up(x), up(r), up(w), up(W)
    so = rb if in_place else up(np.zeros((T, K), np.float32))
    no, lb = up(np.zeros((T, K), np.float32)), up(np.zeros((T, E), np.float32))
    ib, sb = up(np.zeros((T, n_used), np.int32)), up(np.zeros((T, n_used), np.float32))
    rc = ds3.add_rms_norm_router_topk(xb, rb, wb, Wb, so, no, lb, ib, sb, T, K, E, n_used, 1e-6, True)
    assert rc == 0, ds3.last_error()
    s_want, n_want = port.add_rms_norm(x, r, w, 1e-6)
    assert_bitexact(ds3.download(so, np.float32, (T, K)), s_want, "sum")
    got_n = ds3.download(no, np.float32, (T, K))
    assert_close(got_n, n_want, what="norm")
    ref_n = up(np.zeros((T, K), np.float32))
    assert ds3.add_rms_norm(up(x), up(r), wb, None, ref_n, K, T, 1e-6) == 0
    assert_bitexact(got_n, ds3.download(ref_n, np.float32, (T, K)), "norm vs add_rms_norm")
    lg = port.router_logits(got_n, W, 8)
    _, want_i, want_s = port.router(lg, n_used, True)
    assert_bitexact(ds3.download(lb, np.float32, (T, E)), lg, "logits")
    assert_bitexact(ds3.download(ib, np.int32, (T, n_used)), want_i, "top-8")
    assert_close(ds3.download(sb, np.float32, (T, n_used)), want_s, what="scores")


def test_add_rms_norm_router_topk_rejects_other_shapes(ds3, up):
    x = up(I.normal(1, (4, 2080)))
    W = up(I.normal(2, (128, 2080)))
    ib, sb = up(np.zeros((4, 8), np.int32)), up(np.zeros((4, 8), np.float32))
    w = up(I.gamma(2080, 3))
    assert ds3.add_rms_norm_router_topk(x, x, w, W, None, None, None, ib, sb, 4, 2080, 128, 8, 1e-6, True) == -1
    assert "router_logits_topk" in ds3.last_error()
